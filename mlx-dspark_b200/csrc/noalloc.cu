// Verify attention for callers that cannot allocate device memory.
//
// dspark_verify_attn asks its caller for a workspace when a shape splits the keys over more
// CTAs than one thread-block cluster holds (the cross-cluster partial results live there).
// Some callers have no way to provide one: code that is being captured into a CUDA graph, where
// cudaMalloc is not allowed; plugins hosted by a runtime that owns all device memory and hands
// them only their input and output buffers; latency-critical paths that must not take the
// allocator's lock or let a cudaFree synchronize the device. dspark_verify_attn_noalloc serves
// them with the same kernels and a workspace that is a fixed, file-scope device array.
//
// The array is kNoAllocScratchBytes (4 MiB) on every GPU that loads this library, held until the
// process exits. Its host-side name is only a stand-in for the device copy, so the device
// address is looked up once per device (cudaGetSymbolAddress, with that device current) on the
// first call there; that first call should therefore happen before any stream capture. The
// stream must belong to the current device (checked: another device's stream is an argument
// error, since the array's address differs per device). All calls
// on a device share the array: calls that overlap on the GPU (different streams with no ordering
// between them) race on it. Nothing in it needs clearing: every value a launch reads from the
// workspace is written earlier in the same launch sequence.
#include <mutex>

#include "attn.h"
#include "host_common.h"

namespace dspark {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
static __device__ __align__(256) float g_attn_scratch[kNoAllocScratchBytes / sizeof(float)];

constexpr int kMaxDevNoAlloc = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevNoAlloc] = {nullptr};

// Device address of g_attn_scratch on the current device (set up once per device).
int scratch_address(void** out) {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevNoAlloc)
    return fail(DSPARK_ERR_ARG, "verify_attn_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> g(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "verify_attn_noalloc: scratch symbol address");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return DSPARK_OK;
}

}  // namespace
}  // namespace dspark

using namespace dspark;

extern "C" int dspark_verify_attn_noalloc(const void* q, const int64_t q_strides[3], const void* k,
                                          const int64_t k_strides[3], const void* v,
                                          const int64_t v_strides[3], int B, int Hq, int Hk,
                                          int qL, int D, int L, const int32_t* kv_len,
                                          float scale, int causal, const uint32_t* tree_anc,
                                          void* out, const int64_t o_strides[3], void* stream) {
  if (!q || !k || !v || !out || !q_strides || !k_strides || !v_strides || !o_strides)
    return fail(DSPARK_ERR_ARG, "verify_attn_noalloc: null pointer");
  attn::AttnParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_sb = q_strides[0]; p.q_sh = q_strides[1]; p.q_si = q_strides[2];
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.k_sb = k_strides[0]; p.k_sh = k_strides[1]; p.k_ss = k_strides[2];
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.v_sb = v_strides[0]; p.v_sh = v_strides[1]; p.v_ss = v_strides[2];
  p.o = static_cast<__nv_bfloat16*>(out);
  p.o_sb = o_strides[0]; p.o_sh = o_strides[1]; p.o_si = o_strides[2];
  p.kv_len = kv_len;
  p.tree_anc = tree_anc;
  p.B = B; p.Hq = Hq; p.Hk = Hk; p.qL = qL; p.D = D; p.L = L;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  if (B <= 0 || Hk <= 0 || D <= 0 || Hq <= 0 || qL <= 0 || L <= 0)
    return fail(DSPARK_ERR_ARG, "verify_attn_noalloc: bad shape");
  const attn::AttnPlan pl = attn::plan(B, Hq, Hk, qL, D, L);
  const size_t need = attn::workspace_bytes(pl, B, Hk, D);
  if (need > kNoAllocScratchBytes)
    return fail(DSPARK_ERR_UNSUPPORTED,
                "verify_attn_noalloc: this shape needs %zu bytes of scratch, more than the "
                "%zu-byte static maximum (use dspark_verify_attn with a workspace)",
                need, kNoAllocScratchBytes);
  if (need > 0) {
    // the array is looked up for the current device, so the stream must belong to it
    int sdev = -1;
    const cudaError_t se = cudaStreamGetDevice(reinterpret_cast<cudaStream_t>(stream), &sdev);
    if (se != cudaSuccess) return cuda_fail(se, "verify_attn_noalloc: stream device");
    if (sdev != current_device())
      return fail(DSPARK_ERR_ARG,
                  "verify_attn_noalloc: the stream belongs to device %d, the current device is %d",
                  sdev, current_device());
    void* ws = nullptr;
    const int rc = scratch_address(&ws);
    if (rc != DSPARK_OK) return rc;
    p.ws = static_cast<float*>(ws);
  }
  return attn::run(p, &pl, reinterpret_cast<cudaStream_t>(stream));
}
