// Quantized KV cache: the append kernel that quantizes a verify block's new K/V rows into the
// cache (MLX affine, group 64 along head_dim, 4 or 8 bits, bf16 scales / biases), the
// counterpart of mlx-lm's QuantizedKVCache.update_and_fetch used by the reference when kv_bits
// is set (src/mlx_dspark/target.py:166-185). The attention over the quantized cache is the verify
// attention kernel with a dequantizing producer (attn.cu, template parameter QB).
//
// One warp per (row, K or V): lane l holds D/32 consecutive values, a group of 64 values spans
// 64/(D/32) lanes; min / max by shuffles inside the group; the quantization rule is the one
// the build's host quantizer uses (fp32 scale = max((max - min) / (2^bits - 1), 1e-8), bias = min,
// q = round-half-even((x - min) / scale) clamped; scale and bias stored rounded to bf16), so the
// codes are bit-identical to the CPU oracle's. The lanes of one 32-bit code word combine their
// bits by shuffles and the word's first lane stores it.
#include "common.cuh"
#include "host_common.h"

namespace dspark {
namespace kvq {

template <int D, int BITS>
__global__ void __launch_bounds__(64) append_q_kernel(const bf16* kn, int64_t kn_b, int64_t kn_h,
                                                      int64_t kn_t, const bf16* vn, int64_t vn_b,
                                                      int64_t vn_h, int64_t vn_t, dspark_qkv c,
                                                      const int32_t* lens, int cap, int* status) {
  pdl_launch_dependents();
  pdl_wait();
  constexpr int VPL = D / 32;                 // values per lane
  constexpr int GL = 64 / VPL;                // lanes per group (16 or 32)
  constexpr int LPW = 32 / (VPL * BITS);      // lanes per code word
  constexpr float LEVELS = float((1 << BITS) - 1);
  const int t = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = lens[b] + t;
  if (pos < 0 || pos >= cap) {
    if (threadIdx.x == 0) report_error(status, 0x202);
    return;
  }
  const bf16* src = warp == 0 ? kn + b * kn_b + h * kn_h + t * kn_t
                              : vn + b * vn_b + h * vn_h + t * vn_t;
  float x[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) x[i] = bf2f(src[lane * VPL + i]);
  float lo = x[0], hi = x[0];
#pragma unroll
  for (int i = 1; i < VPL; ++i) {
    lo = fminf(lo, x[i]);
    hi = fmaxf(hi, x[i]);
  }
#pragma unroll
  for (int o = 1; o < GL; o <<= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  const float scale = fmaxf((hi - lo) / LEVELS, 1e-8f);
  uint32_t bits = 0;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const float qf = fminf(fmaxf(rintf((x[i] - lo) / scale), 0.f), LEVELS);
    bits |= uint32_t(qf) << (BITS * i);
  }
  // combine LPW lanes into one word: lane j of the word contributes at bit VPL*BITS*j
#pragma unroll
  for (int j = 1; j < LPW; ++j) {
    const uint32_t other = __shfl_down_sync(0xffffffffu, bits, j);
    if ((lane % LPW) == 0) bits |= other << (VPL * BITS * j);
  }
  uint32_t* qrow = (warp == 0 ? c.kq : c.vq) + b * c.q_strides[0] + h * c.q_strides[1] +
                   int64_t(pos) * c.q_strides[2];
  if ((lane % LPW) == 0) qrow[lane / LPW] = bits;
  if ((lane % GL) == 0) {
    const int64_t so = b * c.s_strides[0] + h * c.s_strides[1] + int64_t(pos) * c.s_strides[2] +
                       lane / GL;
    bf16* sp = static_cast<bf16*>(warp == 0 ? c.ks : c.vs);
    bf16* bp = static_cast<bf16*>(warp == 0 ? c.kb : c.vb);
    sp[so] = __float2bfloat16_rn(scale);
    bp[so] = __float2bfloat16_rn(lo);
  }
}

__global__ void lens_add_q_kernel(int32_t* lens, int B, int T, int cap) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) lens[b] = min(cap, lens[b] + T);
}

}  // namespace kvq
}  // namespace dspark

using namespace dspark;

extern "C" int dspark_kv_append_q(const void* k_new, const int64_t kn_strides[3],
                                  const void* v_new, const int64_t vn_strides[3],
                                  const dspark_qkv* cache, int32_t* lens, int B, int H, int T,
                                  int D, int cap, void* stream) {
  if (!k_new || !v_new || !cache || !lens || !kn_strides || !vn_strides)
    return fail(DSPARK_ERR_ARG, "kv_append_q: null pointer");
  const dspark_qkv& c = *cache;
  if (!c.kq || !c.ks || !c.kb || !c.vq || !c.vs || !c.vb)
    return fail(DSPARK_ERR_ARG, "kv_append_q: null cache pointer");
  if (B <= 0 || H <= 0 || T <= 0) return fail(DSPARK_ERR_ARG, "kv_append_q: empty shape");
  if ((D != 64 && D != 128) || (c.bits != 4 && c.bits != 8))
    return fail(DSPARK_ERR_UNSUPPORTED, "kv_append_q: head_dim %d, %d bits (64/128, 4/8)", D, c.bits);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int* st = status_word(current_device());
  const dim3 grid(T, H, B);
  const bf16* kn = static_cast<const bf16*>(k_new);
  const bf16* vn = static_cast<const bf16*>(v_new);
#define DSPARK_APPEND_Q(DD, BB)                                                                 \
  DSPARK_CUDA_TRY(launch_ex(kvq::append_q_kernel<DD, BB>, grid, dim3(64), 0, s, 1, true, kn,   \
                            kn_strides[0], kn_strides[1], kn_strides[2], vn, vn_strides[0],     \
                            vn_strides[1], vn_strides[2], c, (const int32_t*)lens, cap, st),    \
                  "kv_append_q")
  if (D == 128) {
    if (c.bits == 8) DSPARK_APPEND_Q(128, 8); else DSPARK_APPEND_Q(128, 4);
  } else {
    if (c.bits == 8) DSPARK_APPEND_Q(64, 8); else DSPARK_APPEND_Q(64, 4);
  }
#undef DSPARK_APPEND_Q
  DSPARK_CUDA_TRY(launch_ex(kvq::lens_add_q_kernel, dim3((B + 255) / 256), dim3(256), 0, s, 1,
                            true, lens, B, T, cap),
                  "kv_append_q lens");
  return DSPARK_OK;
}
