// Internal interface of the small-M quantized matmul (K1); the C ABI is in include/dspark.h.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dspark {
namespace qmm {

enum Epilogue { EPI_PLAIN = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_QKROPE = 3 };

struct QmmParams {
  const __nv_bfloat16* x = nullptr;  // [M, K] row stride ldx (elements)
  long ldx = 0;
  // segmented rows (an all-gather's [P, M, K/P] output): k lives in segment k / x_seg at
  // x + (k / x_seg) * x_segstride + m * ldx + k % x_seg (x_seg == 0: contiguous rows)
  long x_seg = 0, x_segstride = 0;
  const uint32_t* wq = nullptr;      // [N, K*bits/32]
  const __nv_bfloat16* scales = nullptr;  // [N, K/64]
  const __nv_bfloat16* biases = nullptr;  // [N, K/64]
  const __nv_bfloat16* bias = nullptr;    // optional [N] (EPI_PLAIN)
  __nv_bfloat16* out = nullptr;      // [M, N] row stride ldo (EPI_SWIGLU: [M, N/2])
  long ldo = 0;
  int M = 0, N = 0, K = 0, G = 0, bits = 4;
  // launch geometry (filled from the plan)
  int kslice = 0, cs = 1, nslots = 1;
  int* status = nullptr;
  // prologue RMSNorm of x: rs[m] = rsqrt(sum_e ssq_in[e*ssq_stride+m] / K + eps); x *= rs*norm_w
  const __nv_bfloat16* norm_w = nullptr;
  const float* ssq_in = nullptr;
  int ssq_n = 0;
  int ssq_stride = 32;
  // segmented statistics (an all-gather of per-rank entries): entry e at
  // (e / ssq_seg) * ssq_segstride + (e % ssq_seg) * ssq_stride (ssq_seg == 0: e * ssq_stride)
  int ssq_seg = 0;
  long ssq_segstride = 0;
  float eps = 1e-6f;
  // EPI_RESID: out = bf16(bf16(acc) + resid); ssq_out[ntile*ssq_stride + m] = sum(out^2)
  const __nv_bfloat16* resid = nullptr;
  long ldr = 0;
  float* ssq_out = nullptr;
  // EPI_SWIGLU: number of activation columns (N/2)
  int n_act = 0;
  // EPI_QKROPE: Qwen3 q/k RMSNorm + rotate-half RoPE + KV-cache write (head_dim 128)
  int hq = 0, hk = 0;
  const __nv_bfloat16* qnorm = nullptr;
  const __nv_bfloat16* knorm = nullptr;
  const float* inv_freq = nullptr;   // [64] theta^(-2i/128)
  __nv_bfloat16* qout = nullptr;     // [M, hq*128]
  long ldq = 0;
  __nv_bfloat16* kcache = nullptr;
  __nv_bfloat16* vcache = nullptr;
  int64_t k_sh = 0, k_ss = 0, v_sh = 0, v_ss = 0;  // head / position strides (elements)
  int kv_cap = 0;                    // positions per cache slot (writes at pos >= kv_cap are dropped)
  const int32_t* row_pos = nullptr;  // [M] absolute position of each row
  const int64_t* row_kv = nullptr;   // [M] element offset of the row's cache slot (or null)
  // peer-store epilogue (RESID / SWIGLU, streaming engine): every output element (and RESID
  // statistic) also lands at address + peer_delta[s] for each rank s (peer_delta[own] = 0),
  // and after each tile the writing CTA adds the elements it wrote to *(peer_flag +
  // peer_delta[s]) (release, system scope). peer_world == 0: off.
  int peer_world = 0;
  long peer_delta[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  uint32_t* peer_flag = nullptr;
  // wait before reading x: until wait_flag[s] (s < wait_world) reaches wait_state[0] +
  // wait_elems; the launch's last CTA then advances wait_state[0] (wait_state[1]: CTAs done)
  const uint32_t* wait_flag = nullptr;
  int wait_world = 0;
  uint32_t wait_elems = 0;
  uint32_t* wait_state = nullptr;
};

struct QmmPlan {
  int nw = 0;       // consumer warps; tile width 16*nw output columns
  int cs = 1;       // split-K factor == cluster size
  int kslice = 0;   // k per cluster rank (multiple of 512)
  int nslots = 1;   // pipeline depth
  bool sct = true;  // scales/biases by TMA (needs K % 512 == 0)
  int rt = 2;       // row class the plan was made for (serves M <= 8 * rt)
  int engine = 2;   // 2: streaming (qmm_st.cu); 1: tcgen05 (TMEM operands, qmm_tc.cu);
                    // 0: mma.sync per-tile CTAs (qmm.cu)
  int clusters = 0; // tcgen05: persistent clusters walking the tiles (0: one per cs SMs)
  bool tcmma = false; // streaming engine: tcgen05 MMA consumers (else mma.sync consumers)
  double model_s = 0; // streaming engine: the planner's modelled launch time (seconds)
  // 17-32 rows: run as two launches of the 16-row plan (rows 0-15, then the rest). Chosen for
  // deep-K shapes, where 32 staged rows of x leave shared memory for a high split-K factor only
  // and two 16-row launches are modelled faster. Never set with peer stores or gather waits.
  bool halves = false;
};

// TMA descriptors of the packed weights (128-byte swizzle, boxes of 32 words x tn rows) and,
// when sct, of the scales / biases (boxes of 8 groups x tn rows).
bool tma_maps(const QmmParams& p, int tn, bool sct, CUtensorMap* wmap, CUtensorMap* smap,
              CUtensorMap* bmap);
// tcgen05 engine: geometry and launch (tile 128 rows).
QmmPlan plan_tc(int N, int K, int bits, int rt);
int run_tc(const QmmParams& p, int epi, const QmmPlan& pl, cudaStream_t s);
int tc_smem_bytes(int bits, int rt, int kslice, int nslots);  // layout incl. nslots stages
int tc_stage_bytes(int bits);                                  // one ring stage
int tc_planned_smem(int bits, int rt, int kslice, int nslots); // what a launch requests
int tc_max_clusters(int bits, int rt, int cs, int smem);       // co-resident clusters

// Streaming engine (qmm_st.cu): geometry and launch (tile 128 rows, K % 512 == 0).
QmmPlan plan_st(int N, int K, int bits, int rt);
int run_st(const QmmParams& p, int epi, const QmmPlan& pl, cudaStream_t s);
int st_smem_bytes(int bits, int rt, int kslice, int nslots, int cs, bool tc);
int st_max_clusters(int cs, int smem);

// Geometry for [N, K] at `bits` serving up to 8*rt rows (rt = 2: M <= 16, rt = 4: M <= 32).
// It depends on the weight shape and the row class only, so within a class a row's result
// never depends on how many rows ride with it.
QmmPlan plan(int N, int K, int bits, int epi, int min_tn, int rt = 2);
int run(const QmmParams& p, int epi, const QmmPlan* plan, cudaStream_t stream);

// Wide-M engine (qmm_wide.cu, tcgen05): y = bf16(x . dequant(W)^T) for any M (K % 512 == 0),
// and the full projection (RMSNorm prologue applied to x first, fused epilogue applied to the
// product after) with scratch `ws` of wide_ws_bytes(M, K, N, epi, norm) bytes.
int wide_product(const QmmParams& p, __nv_bfloat16* y, long ldy, cudaStream_t s);
size_t wide_ws_bytes(int M, int K, int N, int epi, bool norm);
int run_wide(const QmmParams& p, int epi, void* ws, size_t ws_bytes, cudaStream_t s);

}  // namespace qmm
}  // namespace dspark
