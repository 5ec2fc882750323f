// C ABI (include/dspark.h): argument checking, host utilities, and the verify-forward layer
// loop that chains the fused kernels on one stream (graph-capturable, programmatic
// dependent launch between consecutive kernels).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <utility>

#include "attn.h"
#include "host_common.h"
#include "ops.h"
#include "qmm.h"

namespace dspark {

static thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(DSPARK_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

static constexpr int kMaxDev = 64;
static int* g_status[kMaxDev] = {nullptr};
static int g_sms[kMaxDev] = {0};
static std::mutex g_mu;

int* status_word(int device) {
  if (device < 0 || device >= kMaxDev) return nullptr;
  return g_status[device];
}

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int sm_count(int device) {
  if (device < 0 || device >= kMaxDev) return 148;
  if (g_sms[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
      n = 148;
    g_sms[device] = n;
  }
  return g_sms[device];
}

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  if (v == nullptr || *v == 0) return dflt;
  return std::atoi(v);
}

bool pdl_enabled() {
  static int on = env_int("DSPARK_PDL", 1);
  return on != 0;
}

static std::atomic<long long> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// Function attributes (dynamic shared memory, cluster size) belong to one device's context, so
// the value a kernel was configured with is kept per (kernel, device).
static std::mutex g_cfg_mu;
static std::map<std::pair<const void*, int>, int> g_cfg;

int configured_value(const void* fn, int device) {
  std::lock_guard<std::mutex> lk(g_cfg_mu);
  auto it = g_cfg.find(std::make_pair(fn, device));
  return it == g_cfg.end() ? 0 : it->second;
}

void set_configured_value(const void* fn, int device, int value) {
  std::lock_guard<std::mutex> lk(g_cfg_mu);
  g_cfg[std::make_pair(fn, device)] = value;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t dim0,
                    uint64_t dim1, uint64_t stride1_bytes, uint32_t box0, uint32_t box1,
                    CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (fn == nullptr) {
    fail(DSPARK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
    return false;
  }
  cuuint64_t dims[2] = {dim0, dim1};
  cuuint64_t strides[1] = {stride1_bytes};
  cuuint32_t box[2] = {box0, box1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    fail(DSPARK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu stride %llu box %u x %u",
         int(r), (unsigned long long)dim0, (unsigned long long)dim1,
         (unsigned long long)stride1_bytes, box0, box1);
    return false;
  }
  return true;
}

bool encode_tmap_nd(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                    const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                    CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (fn == nullptr || rank < 1 || rank > 5) return false;
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    estr[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  return fn(map, dt, cuuint32_t(rank), const_cast<void*>(base), d, st, bx, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ------------------------------------------------------------------------ forward plans

struct PlanKey {
  int dev, N, K, bits, epi;
  bool operator==(const PlanKey& o) const {
    return dev == o.dev && N == o.N && K == o.K && bits == o.bits && epi == o.epi;
  }
};
struct PlanKeyHash {
  size_t operator()(const PlanKey& k) const {
    return (size_t(k.N) * 1000003u) ^ (size_t(k.K) * 7919u) ^ (size_t(k.bits) << 3) ^
           size_t(k.epi) ^ (size_t(k.dev) << 40);
  }
};
static std::unordered_map<PlanKey, qmm::QmmPlan, PlanKeyHash> g_plans;

static qmm::QmmPlan cached_plan(int N, int K, int bits, int epi, int rows) {
  std::lock_guard<std::mutex> lk(g_mu);
  const int rt = rows <= 16 ? 2 : 4;
  PlanKey key{current_device(), N, K, bits, epi * 8 + rt};
  auto it = g_plans.find(key);
  if (it != g_plans.end()) return it->second;
  qmm::QmmPlan pl = qmm::plan(N, K, bits, epi, epi == qmm::EPI_QKROPE ? 128 : 0, rt);
  g_plans[key] = pl;
  return pl;
}

}  // namespace dspark

using namespace dspark;
typedef __nv_bfloat16 bf16;

static inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" {

int dspark_version(void) { return 100; }

const char* dspark_last_error(void) { return g_err.c_str(); }

int dspark_init(int device) {
  if (device < 0 || device >= kMaxDev) return fail(DSPARK_ERR_ARG, "init: bad device %d", device);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_status[device] != nullptr) return DSPARK_OK;
  int prev = 0;
  DSPARK_CUDA_TRY(cudaGetDevice(&prev), "init: get device");
  DSPARK_CUDA_TRY(cudaSetDevice(device), "init: set device");
  int* p = nullptr;
  cudaError_t e = cudaMalloc(&p, 256);
  if (e == cudaSuccess) e = cudaMemset(p, 0, 256);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "init: status word");
  g_status[device] = p;
  sm_count(device);
  return DSPARK_OK;
}

int dspark_set_wait_limit_ns(int device, uint64_t ns) {
  int* w = status_word(device);
  if (w == nullptr) return fail(DSPARK_ERR_NOT_INIT, "set_wait_limit_ns: dspark_init(%d) not called", device);
  int prev = 0;
  DSPARK_CUDA_TRY(cudaGetDevice(&prev), "set_wait_limit_ns");
  DSPARK_CUDA_TRY(cudaSetDevice(device), "set_wait_limit_ns");
  // bytes 8..15 of the status block; 0 restores the built-in bound
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(w + 2, &ns, sizeof(ns), cudaMemcpyHostToDevice);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "set_wait_limit_ns");
  return DSPARK_OK;
}

int dspark_device_status(int device, int* code, int clear) {
  if (code == nullptr) return fail(DSPARK_ERR_ARG, "device_status: null code");
  int* w = status_word(device);
  if (w == nullptr) return fail(DSPARK_ERR_NOT_INIT, "device_status: dspark_init(%d) not called", device);
  int prev = 0;
  DSPARK_CUDA_TRY(cudaGetDevice(&prev), "device_status");
  DSPARK_CUDA_TRY(cudaSetDevice(device), "device_status");
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(code, w, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear) e = cudaMemset(w, 0, sizeof(int));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "device_status");
  return DSPARK_OK;
}

int dspark_sm_count(int device) { return sm_count(device); }

long long dspark_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

// -------------------------------------------------------------------------------- K1

int dspark_qmm_ex(const void* x, int64_t ldx, int M, int K, const uint32_t* wq, const void* scales,
                  const void* biases, const void* bias, int N, int bits, int group, void* out,
                  int64_t ldo, void* stream) {
  if (group != 64) return fail(DSPARK_ERR_UNSUPPORTED, "qmm: group size %d (only 64)", group);
  if (!x || !wq || !scales || !biases || !out) return fail(DSPARK_ERR_ARG, "qmm: null pointer");
  qmm::QmmParams p;
  p.x = static_cast<const bf16*>(x);
  p.ldx = ldx;
  p.M = M;
  p.K = K;
  p.N = N;
  p.bits = bits;
  p.wq = wq;
  p.scales = static_cast<const bf16*>(scales);
  p.biases = static_cast<const bf16*>(biases);
  p.bias = static_cast<const bf16*>(bias);
  p.out = static_cast<bf16*>(out);
  p.ldo = ldo;
  return qmm::run(p, qmm::EPI_PLAIN, nullptr, as_stream(stream));
}

int dspark_qmm(const void* x, int M, int K, const uint32_t* wq, const void* scales,
               const void* biases, int N, int bits, int group, void* out, void* stream) {
  return dspark_qmm_ex(x, K, M, K, wq, scales, biases, nullptr, N, bits, group, out, N, stream);
}

int dspark_qmm_fused(const dspark_qmm_args* a, void* stream) {
  if (!a || !a->x || !a->wq || !a->scales || !a->biases)
    return fail(DSPARK_ERR_ARG, "qmm_fused: null argument");
  if (a->epilogue < qmm::EPI_PLAIN || a->epilogue > qmm::EPI_QKROPE)
    return fail(DSPARK_ERR_ARG, "qmm_fused: epilogue %d", a->epilogue);
  const int epi = a->epilogue;
  if (epi != qmm::EPI_QKROPE && !a->out) return fail(DSPARK_ERR_ARG, "qmm_fused: null out");
  if (epi == qmm::EPI_RESID && !a->resid) return fail(DSPARK_ERR_ARG, "qmm_fused: null resid");
  if (epi == qmm::EPI_QKROPE &&
      (!a->q_out || !a->k_cache || !a->v_cache || !a->row_pos || !a->inv_freq || !a->q_norm ||
       !a->k_norm))
    return fail(DSPARK_ERR_ARG, "qmm_fused: q/k-norm + RoPE epilogue needs its buffers");
  if (a->norm_w && !a->ssq_in) return fail(DSPARK_ERR_ARG, "qmm_fused: norm prologue needs ssq_in");
  qmm::QmmParams p;
  p.x = static_cast<const bf16*>(a->x); p.ldx = a->ldx;
  p.x_seg = a->x_seg; p.x_segstride = a->x_seg_stride;
  p.M = a->M; p.K = a->K; p.N = a->N; p.bits = a->bits;
  p.wq = a->wq;
  p.scales = static_cast<const bf16*>(a->scales);
  p.biases = static_cast<const bf16*>(a->biases);
  p.bias = static_cast<const bf16*>(a->bias);
  p.out = static_cast<bf16*>(a->out); p.ldo = a->ldo;
  p.norm_w = static_cast<const bf16*>(a->norm_w);
  p.ssq_in = a->ssq_in; p.ssq_n = a->ssq_n; p.ssq_stride = a->ssq_stride > 0 ? a->ssq_stride : 32;
  p.ssq_seg = a->ssq_seg; p.ssq_segstride = a->ssq_seg_stride;
  p.eps = a->eps;
  p.resid = static_cast<const bf16*>(a->resid); p.ldr = a->ldr; p.ssq_out = a->ssq_out;
  p.n_act = a->n_act;
  p.hq = a->hq; p.hk = a->hk;
  p.qnorm = static_cast<const bf16*>(a->q_norm);
  p.knorm = static_cast<const bf16*>(a->k_norm);
  p.inv_freq = a->inv_freq;
  p.qout = static_cast<bf16*>(a->q_out); p.ldq = a->ldq;
  p.kcache = static_cast<bf16*>(a->k_cache);
  p.vcache = static_cast<bf16*>(a->v_cache);
  p.k_sh = a->k_sh; p.k_ss = a->k_ss; p.v_sh = a->v_sh; p.v_ss = a->v_ss;
  p.kv_cap = a->kv_cap;
  p.row_pos = a->row_pos; p.row_kv = a->row_kv;
  if (a->peer_world < 0 || a->peer_world > 8 || (a->peer_world > 0 && !a->peer_flag))
    return fail(DSPARK_ERR_ARG, "qmm_fused: peer stores need 1..8 ranks and a flag");
  if (a->peer_world > 0 && epi != qmm::EPI_RESID && epi != qmm::EPI_SWIGLU)
    return fail(DSPARK_ERR_UNSUPPORTED, "qmm_fused: peer stores serve the RESID / SWIGLU epilogues");
  if (a->wait_flag && (a->wait_world < 1 || a->wait_world > 8 || !a->wait_state))
    return fail(DSPARK_ERR_ARG, "qmm_fused: a wait needs 1..8 sources and its state words");
  p.peer_world = a->peer_world;
  for (int s = 0; s < 8; ++s) p.peer_delta[s] = a->peer_delta[s];
  p.peer_flag = a->peer_flag;
  p.wait_flag = a->wait_flag;
  p.wait_world = a->wait_world;
  p.wait_elems = a->wait_elems;
  p.wait_state = a->wait_state;
  if (epi == qmm::EPI_QKROPE) {
    p.out = p.qout;
    p.ldo = 0;
  }
  if (a->M < 1 || a->M > 32) return fail(DSPARK_ERR_UNSUPPORTED, "qmm_fused: M=%d (1..32)", a->M);
  qmm::QmmPlan pl = cached_plan(p.N, p.K, p.bits, epi, a->M);
  return qmm::run(p, epi, &pl, as_stream(stream));
}

int dspark_qmm_wide(const void* x, int64_t ldx, int M, int K, const uint32_t* wq,
                    const void* scales, const void* biases, int N, int bits, void* out,
                    int64_t ldo, void* stream) {
  if (!x || !wq || !scales || !biases || !out) return fail(DSPARK_ERR_ARG, "qmm_wide: null pointer");
  if (ldo < N || ldx < K) return fail(DSPARK_ERR_ARG, "qmm_wide: row strides below the row sizes");
  qmm::QmmParams p;
  p.x = static_cast<const bf16*>(x); p.ldx = ldx; p.M = M; p.K = K; p.N = N; p.bits = bits;
  p.wq = wq;
  p.scales = static_cast<const bf16*>(scales);
  p.biases = static_cast<const bf16*>(biases);
  p.G = K / 64;
  p.status = status_word(current_device());
  return qmm::wide_product(p, static_cast<bf16*>(out), ldo, as_stream(stream));
}

size_t dspark_qmm_wide_workspace(int M, int K, int N, int epilogue, int norm) {
  if (M <= 0 || K <= 0 || N <= 0) return 0;
  return qmm::wide_ws_bytes(M, K, N, epilogue, norm != 0);
}

int dspark_rope_inv_freq(float* inv_freq, int head_dim, float theta, void* stream) {
  if (!inv_freq || head_dim <= 0 || head_dim % 2) return fail(DSPARK_ERR_ARG, "rope_inv_freq: bad args");
  return ops::fill_inv_freq(inv_freq, head_dim, theta, as_stream(stream));
}

int dspark_qmm_plan(int N, int K, int bits, int* tile_n, int* split_k, int* k_slice, int* stages) {
  if (bits != 4 && bits != 8) return fail(DSPARK_ERR_UNSUPPORTED, "qmm_plan: bits %d", bits);
  if (K <= 0 || K % 64 || N <= 0 || N % 8) return fail(DSPARK_ERR_UNSUPPORTED, "qmm_plan: shape");
  qmm::QmmPlan pl = qmm::plan(N, K, bits, qmm::EPI_PLAIN, 0);
  if (pl.nw == 0) return fail(DSPARK_ERR_UNSUPPORTED, "qmm_plan: no geometry");
  if (tile_n) *tile_n = 16 * pl.nw;
  if (split_k) *split_k = pl.cs;
  if (k_slice) *k_slice = pl.kslice;
  if (stages) *stages = pl.nslots;
  return DSPARK_OK;
}

int dspark_qmm_plan_rows(int N, int K, int bits, int rows, int out[7]) {
  if (!out) return fail(DSPARK_ERR_ARG, "qmm_plan_rows: null");
  if (bits != 4 && bits != 8) return fail(DSPARK_ERR_UNSUPPORTED, "qmm_plan_rows: bits %d", bits);
  if (K <= 0 || K % 64 || N <= 0 || N % 8) return fail(DSPARK_ERR_UNSUPPORTED, "qmm_plan_rows: shape");
  if (rows < 1 || rows > 32) return fail(DSPARK_ERR_UNSUPPORTED, "qmm_plan_rows: rows %d", rows);
  const int rt = rows <= 16 ? 2 : 4;
  qmm::QmmPlan pl = qmm::plan(N, K, bits, qmm::EPI_PLAIN, 0, rt);
  if (pl.nw == 0) return fail(DSPARK_ERR_UNSUPPORTED, "qmm_plan_rows: no geometry");
  const bool two = pl.halves && rows > 16;
  if (two) pl = qmm::plan(N, K, bits, qmm::EPI_PLAIN, 0, 2);
  out[0] = 16 * pl.nw; out[1] = pl.cs; out[2] = pl.kslice; out[3] = pl.nslots;
  out[4] = pl.clusters; out[5] = two ? 2 : 1; out[6] = pl.engine;
  return DSPARK_OK;
}

// -------------------------------------------------------------------------------- K2

int dspark_verify_attn_plan(int B, int Hq, int Hk, int qL, int D, int L, int out[6]) {
  if (!out) return fail(DSPARK_ERR_ARG, "verify_attn_plan: null");
  if (B <= 0 || Hk <= 0 || Hq <= 0 || Hq % Hk || qL <= 0 || L <= 0)
    return fail(DSPARK_ERR_ARG, "verify_attn_plan: bad shape");
  attn::AttnPlan pl = attn::plan(B, Hq, Hk, qL, D, L);
  out[0] = pl.nrt; out[1] = pl.ks; out[2] = pl.nrg; out[3] = pl.ns; out[4] = pl.ng; out[5] = pl.chunk;
  return DSPARK_OK;
}

size_t dspark_verify_attn_workspace(int B, int Hq, int Hk, int qL, int D, int L) {
  if (B <= 0 || Hk <= 0 || Hq <= 0 || Hq % Hk || qL <= 0 || L <= 0) return 0;
  attn::AttnPlan pl = attn::plan(B, Hq, Hk, qL, D, L);
  return attn::workspace_bytes(pl, B, Hk, D);
}

int dspark_verify_attn_dt(int dtype, const void* q, const int64_t q_strides[3], const void* k,
                          const int64_t k_strides[3], const void* v, const int64_t v_strides[3],
                          int B, int Hq, int Hk, int qL, int D, int L, const int32_t* kv_len,
                          float scale, int causal, const uint32_t* tree_anc, void* out,
                          const int64_t o_strides[3], void* workspace, size_t ws_bytes,
                          void* stream) {
  if (!q || !k || !v || !out || !q_strides || !k_strides || !v_strides || !o_strides)
    return fail(DSPARK_ERR_ARG, "verify_attn: null pointer");
  if (dtype != DSPARK_DTYPE_BF16 && dtype != DSPARK_DTYPE_F16)
    return fail(DSPARK_ERR_UNSUPPORTED, "verify_attn: dtype %d (bf16 = 0, fp16 = 1)", dtype);
  attn::AttnParams p;
  p.f16 = dtype == DSPARK_DTYPE_F16;
  p.q = static_cast<const bf16*>(q);
  p.q_sb = q_strides[0]; p.q_sh = q_strides[1]; p.q_si = q_strides[2];
  p.k = static_cast<const bf16*>(k);
  p.k_sb = k_strides[0]; p.k_sh = k_strides[1]; p.k_ss = k_strides[2];
  p.v = static_cast<const bf16*>(v);
  p.v_sb = v_strides[0]; p.v_sh = v_strides[1]; p.v_ss = v_strides[2];
  p.o = static_cast<bf16*>(out);
  p.o_sb = o_strides[0]; p.o_sh = o_strides[1]; p.o_si = o_strides[2];
  p.kv_len = kv_len;
  p.tree_anc = tree_anc;
  p.B = B; p.Hq = Hq; p.Hk = Hk; p.qL = qL; p.D = D; p.L = L;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  attn::AttnPlan pl = attn::plan(B, Hq, Hk, qL, D, L);
  const size_t need = attn::workspace_bytes(pl, B, Hk, D);
  if (need > 0) {
    if (workspace == nullptr || ws_bytes < need)
      return fail(DSPARK_ERR_ARG, "verify_attn: needs %zu bytes of workspace (got %zu)", need, ws_bytes);
    p.ws = static_cast<float*>(workspace);
  }
  return attn::run(p, &pl, as_stream(stream));
}

int dspark_verify_attn_q(const void* q, const int64_t q_strides[3], const dspark_qkv* kv, int B,
                         int Hq, int Hk, int qL, int D, int L, const int32_t* kv_len, float scale,
                         int causal, void* out, const int64_t o_strides[3], void* workspace,
                         size_t ws_bytes, void* stream) {
  if (!q || !kv || !out || !q_strides || !o_strides)
    return fail(DSPARK_ERR_ARG, "verify_attn_q: null pointer");
  attn::AttnParams p;
  p.q = static_cast<const bf16*>(q);
  p.q_sb = q_strides[0]; p.q_sh = q_strides[1]; p.q_si = q_strides[2];
  p.o = static_cast<bf16*>(out);
  p.o_sb = o_strides[0]; p.o_sh = o_strides[1]; p.o_si = o_strides[2];
  p.qbits = kv->bits;
  p.kq = kv->kq; p.vq = kv->vq;
  p.ksc = static_cast<const bf16*>(kv->ks); p.kbi = static_cast<const bf16*>(kv->kb);
  p.vsc = static_cast<const bf16*>(kv->vs); p.vbi = static_cast<const bf16*>(kv->vb);
  p.kq_sb = kv->q_strides[0]; p.kq_sh = kv->q_strides[1]; p.kq_ss = kv->q_strides[2];
  p.ks_sb = kv->s_strides[0]; p.ks_sh = kv->s_strides[1]; p.ks_ss = kv->s_strides[2];
  p.kv_len = kv_len;
  p.B = B; p.Hq = Hq; p.Hk = Hk; p.qL = qL; p.D = D; p.L = L;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  attn::AttnPlan pl = attn::plan(B, Hq, Hk, qL, D, L);
  if (D > 128) return fail(DSPARK_ERR_UNSUPPORTED, "verify_attn_q: head_dim %d (64, 128)", D);
  const size_t need = attn::workspace_bytes(pl, B, Hk, D);
  if (need > 0) {
    if (workspace == nullptr || ws_bytes < need)
      return fail(DSPARK_ERR_ARG, "verify_attn_q: needs %zu bytes of workspace (got %zu)", need, ws_bytes);
    p.ws = static_cast<float*>(workspace);
  }
  return attn::run(p, &pl, as_stream(stream));
}

int dspark_verify_attn(const void* q, const int64_t q_strides[3], const void* k,
                       const int64_t k_strides[3], const void* v, const int64_t v_strides[3],
                       int B, int Hq, int Hk, int qL, int D, int L, const int32_t* kv_len,
                       float scale, int causal, const uint32_t* tree_anc, void* out,
                       const int64_t o_strides[3], void* workspace, size_t ws_bytes,
                       void* stream) {
  return dspark_verify_attn_dt(DSPARK_DTYPE_BF16, q, q_strides, k, k_strides, v, v_strides, B,
                               Hq, Hk, qL, D, L, kv_len, scale, causal, tree_anc, out, o_strides,
                               workspace, ws_bytes, stream);
}

int dspark_verify_attn_ragged(const void* q, int64_t q_sh, int64_t q_si, const void* k,
                              int64_t k_sh, int64_t k_ss, const void* v, int64_t v_sh,
                              int64_t v_ss, const int32_t* row_start, const int32_t* q_len,
                              const int64_t* kv_off, const int32_t* kv_len, int B, int Hq,
                              int Hk, int qL_max, int D, int L_max, float scale, void* out,
                              int64_t o_sh, int64_t o_si, void* workspace, size_t ws_bytes,
                              void* stream) {
  if (!q || !k || !v || !out || !row_start || !q_len || !kv_off || !kv_len)
    return fail(DSPARK_ERR_ARG, "verify_attn_ragged: null pointer");
  attn::AttnParams p;
  p.q = static_cast<const bf16*>(q);
  p.q_sh = q_sh; p.q_si = q_si;
  p.k = static_cast<const bf16*>(k);
  p.k_sh = k_sh; p.k_ss = k_ss;
  p.v = static_cast<const bf16*>(v);
  p.v_sh = v_sh; p.v_ss = v_ss;
  p.o = static_cast<bf16*>(out);
  p.o_sh = o_sh; p.o_si = o_si;
  p.row_start = row_start; p.q_len = q_len; p.kv_off = kv_off; p.kv_len = kv_len;
  p.B = B; p.Hq = Hq; p.Hk = Hk; p.qL = qL_max; p.D = D; p.L = L_max;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = 1;
  attn::AttnPlan pl = attn::plan(B, Hq, Hk, qL_max, D, L_max);
  const size_t need = attn::workspace_bytes(pl, B, Hk, D);
  if (need > 0) {
    if (workspace == nullptr || ws_bytes < need)
      return fail(DSPARK_ERR_ARG, "verify_attn_ragged: needs %zu bytes of workspace", need);
    p.ws = static_cast<float*>(workspace);
  }
  return attn::run(p, &pl, as_stream(stream));
}

// -------------------------------------------------------------------------------- K3/K4

int dspark_kv_append(const void* k_new, const int64_t kn_strides[3], const void* v_new,
                     const int64_t vn_strides[3], void* k_cache, const int64_t kc_strides[3],
                     void* v_cache, const int64_t vc_strides[3], int32_t* lens, int B, int H,
                     int T, int D, int elem_size, int cap, void* stream) {
  if (!k_new || !v_new || !k_cache || !v_cache || !lens) return fail(DSPARK_ERR_ARG, "kv_append: null");
  if (elem_size != 1 && elem_size != 2 && elem_size != 4 && elem_size != 8)
    return fail(DSPARK_ERR_ARG, "kv_append: element size %d", elem_size);
  ops::KvAppend a;
  a.kn = k_new;
  a.vn = v_new;
  a.kc = k_cache;
  a.vc = v_cache;
  for (int i = 0; i < 3; ++i) {
    a.kn_s[i] = kn_strides[i];
    a.vn_s[i] = vn_strides[i];
    a.kc_s[i] = kc_strides[i];
    a.vc_s[i] = vc_strides[i];
  }
  a.lens = lens;
  a.B = B; a.H = H; a.T = T; a.D = D; a.cap = cap; a.esize = elem_size;
  return ops::kv_append(a, as_stream(stream));
}

int dspark_kv_rollback(int32_t* lens, const int32_t* n_rejected, int B, void* stream) {
  if (!lens || !n_rejected) return fail(DSPARK_ERR_ARG, "kv_rollback: null");
  return ops::kv_rollback(lens, n_rejected, B, as_stream(stream));
}

int dspark_kv_move_row(void* k_cache, const int64_t kc_strides[3], void* v_cache,
                       const int64_t vc_strides[3], int32_t* lens, int src, int dst, int H, int D,
                       int elem_size, int max_len, void* stream) {
  if (!k_cache || !v_cache || !lens) return fail(DSPARK_ERR_ARG, "kv_move_row: null");
  if (elem_size != 1 && elem_size != 2 && elem_size != 4 && elem_size != 8)
    return fail(DSPARK_ERR_ARG, "kv_move_row: element size %d", elem_size);
  return ops::kv_move_row(k_cache, kc_strides, v_cache, vc_strides, lens, src, dst, H, D,
                          elem_size, max_len, as_stream(stream));
}

int dspark_argmax(const void* logits, int64_t ld, int R, int V, int32_t* tt, void* stream) {
  if (!logits || !tt) return fail(DSPARK_ERR_ARG, "argmax: null");
  return ops::argmax(static_cast<const bf16*>(logits), ld, R, V, tt, as_stream(stream));
}

int dspark_accept(const int32_t* tt, const int32_t* ids, const int32_t* cu_rows, int B,
                  int32_t* n_accept, int32_t* next_tok, int32_t* lens, void* stream) {
  if (!tt || !ids || !cu_rows) return fail(DSPARK_ERR_ARG, "accept: null");
  return ops::accept(tt, ids, cu_rows, B, n_accept, next_tok, lens, as_stream(stream));
}

int dspark_pack_ragged(const int32_t* block_len, const int32_t* kv_len, const int64_t* slot_off,
                       const int32_t* ids_pad, int t_max, int B, int r_max, int32_t* cu_rows,
                       int32_t* row_pos, int64_t* row_kv, int32_t* row_req, int32_t* ids,
                       int32_t* kv_len_new, void* stream) {
  if (!block_len || !kv_len || !slot_off || !ids_pad || !cu_rows || !row_pos || !row_kv ||
      !row_req || !ids || !kv_len_new)
    return fail(DSPARK_ERR_ARG, "pack_ragged: null");
  return ops::pack_ragged(block_len, kv_len, slot_off, ids_pad, t_max, B, r_max, cu_rows, row_pos,
                          row_kv, row_req, ids, kv_len_new, as_stream(stream));
}

int dspark_batch_mask(const int32_t* offsets, int B, int T, int Lcur, uint8_t* mask, void* stream) {
  if (!offsets || !mask) return fail(DSPARK_ERR_ARG, "batch_mask: null");
  return ops::batch_mask(offsets, B, T, Lcur, mask, as_stream(stream));
}

int dspark_embed(const int32_t* ids, int M, const uint32_t* wq, const void* scales,
                 const void* biases, int V, int H, int bits, void* h, float* ssq, void* stream) {
  if (!ids || !wq || !scales || !biases || !h) return fail(DSPARK_ERR_ARG, "embed: null");
  return ops::embed(ids, M, wq, static_cast<const bf16*>(scales), static_cast<const bf16*>(biases),
                    H, V, bits, static_cast<bf16*>(h), ssq, as_stream(stream));
}

int dspark_rmsnorm(const void* x, int64_t ldx, int M, int H, const void* w, float eps, void* out,
                   int64_t ldo, void* stream) {
  if (!x || !w || !out) return fail(DSPARK_ERR_ARG, "rmsnorm: null");
  return ops::rmsnorm(static_cast<const bf16*>(x), ldx, M, H, static_cast<const bf16*>(w), eps,
                      static_cast<bf16*>(out), ldo, as_stream(stream));
}

int dspark_verify_prepare(int32_t* len, int R, const dspark_fwd_buffers* b, void* stream) {
  if (!len || !b) return fail(DSPARK_ERR_ARG, "verify_prepare: null");
  return ops::verify_prepare(len, R, b->row_pos, b->row_kv, b->kv_len, b->row_start, b->q_len,
                             b->kv_off, as_stream(stream));
}

// -------------------------------------------------------------------------------- forward

#define DSPARK_TRY(expr)              \
  do {                                \
    int _rc = (expr);                 \
    if (_rc != DSPARK_OK) return _rc; \
  } while (0)

int dspark_verify_forward(const dspark_model* m, const dspark_fwd_buffers* buf, const int32_t* ids,
                          int R, int B, int qL_max, int L_max, void* logits, int64_t ld_logits,
                          void* stream) {
  if (!m || !buf || !ids || !logits || !m->layers) return fail(DSPARK_ERR_ARG, "forward: null");
  if (m->head_dim != 128) return fail(DSPARK_ERR_UNSUPPORTED, "forward: head_dim %d (needs 128)", m->head_dim);
  const int rows_cap = buf->rows_cap > 0 ? buf->rows_cap : 32;
  if (R < 1 || R > rows_cap) return fail(DSPARK_ERR_UNSUPPORTED, "forward: R=%d rows (1..%d)", R, rows_cap);
  if (qL_max < 1 || qL_max > 32) return fail(DSPARK_ERR_UNSUPPORTED, "forward: qL_max=%d (1..32)", qL_max);
  if (m->hidden % 512 || m->intermediate % 512)
    return fail(DSPARK_ERR_UNSUPPORTED, "forward: hidden / intermediate must be multiples of 512");
  cudaStream_t s = as_stream(stream);
  const int H = m->hidden, D = m->head_dim, Hq = m->n_heads, Hk = m->n_kv_heads;
  const int I = m->intermediate;
  bf16* h = static_cast<bf16*>(buf->h);
  bf16* xq = static_cast<bf16*>(buf->xq);
  bf16* at = static_cast<bf16*>(buf->attn);
  bf16* act = static_cast<bf16*>(buf->act);
  const int kSsqStride = rows_cap;  // statistics entry e of row m at e * kSsqStride + m
  // many rows: every projection runs once over all R rows in the wide-M engine, given its scratch
  const int wide_min = env_int("DSPARK_WIDE_MIN_ROWS", 64);
  bool wide = R >= wide_min && buf->wide_ws != nullptr;
  if (wide) {
    size_t need = 0;
    for (int l = 0; l < m->n_layers; ++l) {
      const dspark_layer& L = m->layers[l];
      need = std::max({need, qmm::wide_ws_bytes(R, H, L.qkv.N, qmm::EPI_QKROPE, true),
                       qmm::wide_ws_bytes(R, L.o.K, L.o.N, qmm::EPI_RESID, false),
                       qmm::wide_ws_bytes(R, H, L.gate_up.N, qmm::EPI_SWIGLU, true),
                       qmm::wide_ws_bytes(R, L.down.K, L.down.N, qmm::EPI_RESID, false)});
    }
    need = std::max(need, qmm::wide_ws_bytes(R, H, m->lm_head.N, qmm::EPI_PLAIN, true));
    wide = need <= buf->wide_ws_bytes;
  }
  const int kChunk = wide ? R : 32;  // rows per projection launch

  DSPARK_TRY(ops::fill_inv_freq(buf->inv_freq, D, m->rope_theta, s));
  DSPARK_TRY(ops::embed(ids, R, m->embed.wq, static_cast<const bf16*>(m->embed.scales),
                        static_cast<const bf16*>(m->embed.biases), H, m->embed.N, m->embed.bits, h,
                        buf->ssq_a, s));
  int ssq_n = 1;  // entries of the current statistics buffer
  float* ssq_cur = buf->ssq_a;

  for (int l = 0; l < m->n_layers; ++l) {
    const dspark_layer& L = m->layers[l];
    // fused QKV projection + input RMSNorm + q/k RMSNorm + RoPE + cache write
    for (int r0 = 0; r0 < R; r0 += kChunk) {
      const int mr = std::min(kChunk, R - r0);
      qmm::QmmParams p;
      p.x = h + int64_t(r0) * H; p.ldx = H; p.M = mr; p.K = H; p.N = L.qkv.N; p.bits = L.qkv.bits;
      p.wq = L.qkv.wq;
      p.scales = static_cast<const bf16*>(L.qkv.scales);
      p.biases = static_cast<const bf16*>(L.qkv.biases);
      p.norm_w = static_cast<const bf16*>(L.in_norm);
      p.ssq_in = ssq_cur + r0; p.ssq_n = ssq_n; p.ssq_stride = kSsqStride; p.eps = m->rms_eps;
      p.hq = Hq; p.hk = Hk;
      p.qnorm = static_cast<const bf16*>(L.q_norm);
      p.knorm = static_cast<const bf16*>(L.k_norm);
      p.inv_freq = buf->inv_freq;
      p.qout = xq + int64_t(r0) * Hq * D; p.ldq = int64_t(Hq) * D;
      p.kcache = static_cast<bf16*>(L.k_cache);
      p.vcache = static_cast<bf16*>(L.v_cache);
      p.k_sh = m->k_sh; p.k_ss = m->k_ss; p.v_sh = m->v_sh; p.v_ss = m->v_ss;
      p.kv_cap = m->kv_cap;
      p.row_pos = buf->row_pos + r0; p.row_kv = buf->row_kv + r0;
      p.out = xq; p.ldo = 0;
      if (wide) {
        DSPARK_TRY(qmm::run_wide(p, qmm::EPI_QKROPE, buf->wide_ws, buf->wide_ws_bytes, s));
      } else {
        qmm::QmmPlan pl = cached_plan(p.N, p.K, p.bits, qmm::EPI_QKROPE, mr);
        DSPARK_TRY(qmm::run(p, qmm::EPI_QKROPE, &pl, s));
      }
    }
    // verify attention over each request's cache slot
    {
      attn::AttnParams a;
      a.q = xq; a.q_sh = D; a.q_si = int64_t(Hq) * D;
      a.o = at; a.o_sh = D; a.o_si = int64_t(Hq) * D;
      a.k = static_cast<const bf16*>(L.k_cache); a.k_sh = m->k_sh; a.k_ss = m->k_ss;
      a.v = static_cast<const bf16*>(L.v_cache); a.v_sh = m->v_sh; a.v_ss = m->v_ss;
      a.row_start = buf->row_start; a.q_len = buf->q_len; a.kv_off = buf->kv_off;
      a.kv_len = buf->kv_len;
      a.B = B; a.Hq = Hq; a.Hk = Hk; a.qL = qL_max; a.D = D; a.L = L_max;
      a.scale_log2 = (1.0f / std::sqrt(float(D))) * 1.4426950408889634f;
      a.causal = 1;
      attn::AttnPlan apl = attn::plan(B, Hq, Hk, qL_max, D, L_max);
      if (attn::workspace_bytes(apl, B, Hk, D) > buf->attn_ws_bytes) {
        // not enough workspace: stay within one cluster group
        apl.ng = 1;
        apl.chunk = ((L_max + apl.ns - 1) / apl.ns + 63) / 64 * 64;
      }
      a.ws = static_cast<float*>(buf->attn_ws);
      DSPARK_TRY(attn::run(a, &apl, s));
    }
    // O projection + residual (in place on h) + statistics for the post-attention norm
    int ssq_n_b = 0;
    for (int r0 = 0; r0 < R; r0 += kChunk) {
      const int mr = std::min(kChunk, R - r0);
      qmm::QmmParams p;
      p.x = at + int64_t(r0) * Hq * D; p.ldx = int64_t(Hq) * D; p.M = mr; p.K = Hq * D;
      p.N = L.o.N; p.bits = L.o.bits;
      p.wq = L.o.wq;
      p.scales = static_cast<const bf16*>(L.o.scales);
      p.biases = static_cast<const bf16*>(L.o.biases);
      p.resid = h + int64_t(r0) * H; p.ldr = H; p.out = h + int64_t(r0) * H; p.ldo = H;
      p.ssq_out = buf->ssq_b + r0; p.ssq_stride = kSsqStride;
      if (wide) {
        ssq_n_b = (p.N + 127) / 128;  // one statistics entry per 128-column epilogue tile
        DSPARK_TRY(qmm::run_wide(p, qmm::EPI_RESID, buf->wide_ws, buf->wide_ws_bytes, s));
      } else {
        qmm::QmmPlan pl = cached_plan(p.N, p.K, p.bits, qmm::EPI_RESID, mr);
        ssq_n_b = pl.nw > 0 ? (p.N + 16 * pl.nw - 1) / (16 * pl.nw) : 0;  // run() rejects nw == 0
        DSPARK_TRY(qmm::run(p, qmm::EPI_RESID, &pl, s));
      }
    }
    // gate/up projection + post-attention RMSNorm + SwiGLU
    for (int r0 = 0; r0 < R; r0 += kChunk) {
      const int mr = std::min(kChunk, R - r0);
      qmm::QmmParams p;
      p.x = h + int64_t(r0) * H; p.ldx = H; p.M = mr; p.K = H; p.N = L.gate_up.N;
      p.bits = L.gate_up.bits;
      p.wq = L.gate_up.wq;
      p.scales = static_cast<const bf16*>(L.gate_up.scales);
      p.biases = static_cast<const bf16*>(L.gate_up.biases);
      p.norm_w = static_cast<const bf16*>(L.post_norm);
      p.ssq_in = buf->ssq_b + r0; p.ssq_n = ssq_n_b; p.ssq_stride = kSsqStride; p.eps = m->rms_eps;
      p.out = act + int64_t(r0) * I; p.ldo = I; p.n_act = I;
      if (wide) {
        DSPARK_TRY(qmm::run_wide(p, qmm::EPI_SWIGLU, buf->wide_ws, buf->wide_ws_bytes, s));
      } else {
        qmm::QmmPlan pl = cached_plan(p.N, p.K, p.bits, qmm::EPI_SWIGLU, mr);
        DSPARK_TRY(qmm::run(p, qmm::EPI_SWIGLU, &pl, s));
      }
    }
    // down projection + residual + statistics for the next input norm
    for (int r0 = 0; r0 < R; r0 += kChunk) {
      const int mr = std::min(kChunk, R - r0);
      qmm::QmmParams p;
      p.x = act + int64_t(r0) * I; p.ldx = I; p.M = mr; p.K = I; p.N = L.down.N; p.bits = L.down.bits;
      p.wq = L.down.wq;
      p.scales = static_cast<const bf16*>(L.down.scales);
      p.biases = static_cast<const bf16*>(L.down.biases);
      p.resid = h + int64_t(r0) * H; p.ldr = H; p.out = h + int64_t(r0) * H; p.ldo = H;
      p.ssq_out = buf->ssq_a + r0; p.ssq_stride = kSsqStride;
      if (wide) {
        ssq_n = (p.N + 127) / 128;
        DSPARK_TRY(qmm::run_wide(p, qmm::EPI_RESID, buf->wide_ws, buf->wide_ws_bytes, s));
      } else {
        qmm::QmmPlan pl = cached_plan(p.N, p.K, p.bits, qmm::EPI_RESID, mr);
        ssq_n = pl.nw > 0 ? (p.N + 16 * pl.nw - 1) / (16 * pl.nw) : 0;  // run() rejects nw == 0
        DSPARK_TRY(qmm::run(p, qmm::EPI_RESID, &pl, s));
      }
    }
    ssq_cur = buf->ssq_a;
  }
  // final RMSNorm + lm_head
  for (int r0 = 0; r0 < R; r0 += kChunk) {
    const int mr = std::min(kChunk, R - r0);
    qmm::QmmParams p;
    p.x = h + int64_t(r0) * H; p.ldx = H; p.M = mr; p.K = H; p.N = m->lm_head.N;
    p.bits = m->lm_head.bits;
    p.wq = m->lm_head.wq;
    p.scales = static_cast<const bf16*>(m->lm_head.scales);
    p.biases = static_cast<const bf16*>(m->lm_head.biases);
    p.norm_w = static_cast<const bf16*>(m->final_norm);
    p.ssq_in = ssq_cur + r0; p.ssq_n = ssq_n; p.ssq_stride = kSsqStride; p.eps = m->rms_eps;
    p.out = static_cast<bf16*>(logits) + int64_t(r0) * ld_logits; p.ldo = ld_logits;
    if (wide) {
      DSPARK_TRY(qmm::run_wide(p, qmm::EPI_PLAIN, buf->wide_ws, buf->wide_ws_bytes, s));
    } else {
      qmm::QmmPlan pl = cached_plan(p.N, p.K, p.bits, qmm::EPI_PLAIN, mr);
      DSPARK_TRY(qmm::run(p, qmm::EPI_PLAIN, &pl, s));
    }
  }
  return DSPARK_OK;
}

}  // extern "C"
