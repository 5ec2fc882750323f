// K1, wide-M engine: y[M, N] = bf16(x[M, K] . dequant(W)^T) for many rows (prefill-width
// calls and the batch engine's packed verify rows) on the 5th-generation tensor cores, plus the
// two small kernels that let the verify forward's fused projections use it: the RMSNorm
// prologue applied once to x, and the shared epilogues (residual + statistics, SwiGLU, q/k-norm
// + RoPE + KV write) applied to the bf16 product.
//
// Counterpart of src/mlx_dspark/wide_gemm.py (x @ mx.dequantize(w).T above a row threshold): the
// weights are dequantized once per tile into tensor memory and reused by 256 x rows, instead of
// the small-M engines' per-32-row launches that each re-read every weight.
//
// Per CTA (persistent over tiles t = (weight tile, x tile), 1 CTA per SM):
//  * producer warp: TMA per 64-k stage — x [256 rows x 64 k] bf16 with the 128-byte swizzle (the
//    UMMA K-major canonical layout, read by the tensor core as the B operand), the packed
//    weights [128 rows x 64 k], and every 8 stages the bf16 scales / biases of 8 groups;
//  * four dequantization warps: thread r of the warpgroup owns weight row r == TMEM lane r and
//    writes its 64 weights of the stage, w = scale * q + bias rounded once to bf16 (q exact from
//    the magic-exponent extraction: nibble | 0x4300 = 128 + q, minus 128; 8-bit as two nibble
//    planes, q = lo + 16 hi exactly), in natural k order into one of four A buffers in tensor
//    memory (32 columns of bf16 pairs);
//  * one MMA warp: per stage 4 MMAs kind::f16 (M = 128 weight rows from tensor memory, N = 256
//    x rows from shared memory, K = 16) accumulate the tile into D (256 fp32 columns); commits
//    free the A buffer and the ring slot, and hand D to the epilogue warps at the tile's end;
//  * four epilogue warps: read D (lane = weight row n, column = x row m) and store bf16(D) at
//    y[m, n] (each warp's 32 lanes write 64 contiguous bytes per row m).
// On B200 a kind::f16 MMA with M = 128, K = 16 costs ~100 cycles up to N = 128 and ~145 at
// N = 256 (microbenchmark), so N = 256 keeps the tensor core near its peak rate.
// Every mbarrier wait is time-bounded (the device status word records a wait that ran out).
#include <algorithm>

#include "common.cuh"
#include "host_common.h"
#include "qmm.h"
#include "qmm_epilogue.cuh"
#include "tcgen05.cuh"

namespace dspark {
namespace qmm {
namespace wide {

constexpr int TN = 128;             // weight rows per tile (MMA M, TMEM lanes)
constexpr int TX = 256;             // x rows per tile (MMA N)
constexpr int KS = 64;              // k per stage (one quantization group)
constexpr int NST = 4;              // ring stages
constexpr int NA = 4;               // A buffers in tensor memory
constexpr int NSC = 2;              // scale-block slots (8 groups each)
constexpr int XSTG = TX * 128;      // x tile of a stage: 256 rows x 128 bytes
constexpr int SCB = TN * 16;        // 8 groups of bf16 scales (or biases) for 128 rows
constexpr int WARP_TMA = 0, WARP_MMA = 1, WARP_DQ = 2, WARP_EPI = 6;
constexpr int NTHR = 10 * 32;
constexpr uint32_t DCOL = 256;      // D: tensor-memory columns 256 .. 511
constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(TX >> 3) << 17) |
                           (uint32_t(TN >> 4) << 24);  // bf16 x bf16 -> f32, K-major, 128 x 256

template <int BITS>
__host__ __device__ constexpr int wstg() { return TN * KS * BITS / 8; }  // 4 or 8 KB

struct Layout {
  int xr, wr, sr, bars, total;
};

template <int BITS>
__host__ __device__ constexpr Layout layout() {
  Layout L{};
  int off = 0;
  L.xr = off;                       // 1024-byte aligned (128-byte swizzle atoms)
  off += NST * XSTG;
  L.wr = off;
  off += NST * wstg<BITS>();
  L.sr = off;
  off += NSC * 2 * SCB;
  L.bars = off;
  off += (2 * NST + 2 * NA + 3) * 8 + 16;
  L.total = off + 1024;             // slack to align the dynamic base
  return L;
}

// Shared-memory matrix descriptor of a K-major operand with the 128-byte swizzle (8-row groups
// 1024 bytes apart; the leading offset is unused for swizzled K-major layouts).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFF);
  d |= uint64_t(1) << 16;
  d |= uint64_t(1024 >> 4) << 32;
  d |= uint64_t(1) << 46;           // descriptor version (sm_100)
  d |= uint64_t(2) << 61;           // 128-byte swizzle
  return d;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint32_t bf2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t dup_group(uint4 v, int g) {
  const int w = g >> 1;
  const uint32_t x = w == 0 ? v.x : w == 1 ? v.y : w == 2 ? v.z : v.w;
  return __byte_perm(x, 0u, (g & 1) ? 0x3232u : 0x1010u);
}

struct WideArgs {
  long ldy = 0;
  __nv_bfloat16* y = nullptr;
  int ntm = 0, ntiles = 0;
  int* status = nullptr;
  int M = 0, N = 0, K = 0;
};

template <int BITS>
__global__ void __launch_bounds__(NTHR, 1)
    wide_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                const __grid_constant__ CUtensorMap smap, const __grid_constant__ CUtensorMap bmap,
                const WideArgs a) {
  constexpr Layout Lo = layout<BITS>();
  constexpr int WSTG = wstg<BITS>();
  constexpr uint32_t M128 = 0x43004300u;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align_up<1024>(smem_raw);
  uint8_t* xr = smem + Lo.xr;
  uint8_t* wr = smem + Lo.wr;
  uint8_t* sr = smem + Lo.sr;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lo.bars);
  uint64_t* empty = full + NST;
  uint64_t* afull = empty + NST;
  uint64_t* aempty = afull + NA;
  uint64_t* dfull = aempty + NA;
  uint64_t* dempty = dfull + 1;
  uint64_t* mfin = dempty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mfin + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = a.K / KS;  // stages per tile
  if (warp == WARP_TMA && lane == 0) {
    prefetch_tmap(&xmap);
    prefetch_tmap(&wmap);
    prefetch_tmap(&smap);
    prefetch_tmap(&bmap);
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4 + 1);  // the dequantization warps + the MMA warp's commit
    }
    for (int i = 0; i < NA; ++i) {
      mbar_init(&afull[i], 4);
      mbar_init(&aempty[i], 1);
    }
    mbar_init(dfull, 1);
    mbar_init(dempty, 4);
    mbar_init(mfin, 1);
    fence_mbar_init();
  }
  if (warp == 0) tcg::tmem_alloc(tmem_slot, 512);
  tcg::tc_fence_before();
  __syncthreads();
  tcg::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  bool ok = true;
  if (warp == WARP_TMA) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      pdl_wait();  // x comes from the previous kernel
      const uint64_t keep = l2_policy_evict_last();  // x is re-read by every weight tile
      int g = 0, sb = 0;
      for (int t = blockIdx.x; t < a.ntiles && ok; t += gridDim.x) {
        const int n0 = (t / a.ntm) * TN, m0 = (t % a.ntm) * TX;
        for (int st = 0; st < nk; ++st, ++g) {
          const int slot = g % NST;
          if (g >= NST && !(ok = mbar_wait(&empty[slot], uint32_t(((g / NST) - 1) & 1), a.status,
                                           kErrWaitEmpty)))
            break;
          const bool sblk = (st & 7) == 0;
          mbar_arrive_expect_tx(&full[slot], XSTG + WSTG + (sblk ? 2 * SCB : 0));
          tma_load_2d(xr + slot * XSTG, &xmap, &full[slot], st * KS, m0, keep);
          tma_load_2d(wr + slot * WSTG, &wmap, &full[slot], st * (KS * BITS / 32), n0, keep);
          if (sblk) {
            const int ss = sb % NSC;
            tma_load_2d(sr + ss * 2 * SCB, &smap, &full[slot], st, n0, keep);
            tma_load_2d(sr + ss * 2 * SCB + SCB, &bmap, &full[slot], st, n0, keep);
            ++sb;
          }
        }
      }
      // no copy may still be in flight when the CTA exits
      for (int i = max(0, g - NST); i < g; ++i)
        mbar_wait(&full[i % NST], uint32_t((i / NST) & 1), a.status, kErrWaitFull);
    }
    __syncwarp();
  } else if (warp == WARP_MMA) {
    // ---------------------------------------------------------------- MMA issue
    if (tcg::elect_one()) {
      int g = 0, j = 0;
      bool issued = false;
      for (int t = blockIdx.x; t < a.ntiles && ok; t += gridDim.x, ++j) {
        if (j >= 1) ok = mbar_wait(dempty, uint32_t((j - 1) & 1), a.status, kErrWaitMma);
        tcg::tc_fence_after();
        for (int st = 0; st < nk && ok; ++st, ++g) {
          const int slot = g % NST, ab = g % NA;
          ok = mbar_wait(&full[slot], uint32_t((g / NST) & 1), a.status, kErrWaitFull);
          if (ok) ok = mbar_wait(&afull[ab], uint32_t((g / NA) & 1), a.status, kErrWaitMma);
          if (!ok) break;
          tcg::tc_fence_after();
          const uint64_t bd = desc_sw128(smem_u32(xr + slot * XSTG));
#pragma unroll
          for (int s = 0; s < KS / 16; ++s)
            tcg::umma_ts(tmem + DCOL, tmem + uint32_t(ab * 32 + 8 * s), bd + uint64_t(2 * s),
                         IDESC, (st | s) ? 1u : 0u);
          tcg::umma_commit(&aempty[ab]);
          tcg::umma_commit(&empty[slot]);
          issued = true;
        }
        if (ok) tcg::umma_commit(dfull);
      }
      if (issued) {  // nothing may write tensor memory after the CTA releases it
        tcg::umma_commit(mfin);
        mbar_wait(mfin, 0, a.status, kErrWaitMma);
      }
    }
    __syncwarp();
  } else if (warp < WARP_EPI) {
    // ---------------------------------------------------------------- dequantization
    const int q = warp & 3, row = q * 32 + lane;
    const uint32_t ta = tmem + (uint32_t(q * 32) << 16);
    const uint32_t wr_a = smem_u32(wr), sr_a = smem_u32(sr);
    int g = 0, sb = 0;
    uint4 sv4 = make_uint4(0u, 0u, 0u, 0u), bv4 = sv4;
    for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x) {
      for (int st = 0; st < nk; ++st, ++g) {
        const int slot = g % NST, ab = g % NA;
        if (ok) ok = mbar_wait(&full[slot], uint32_t((g / NST) & 1), a.status, kErrWaitFull);
        if ((st & 7) == 0) {
          const uint32_t sa = sr_a + uint32_t((sb % NSC) * 2 * SCB + row * 16);
          sv4 = lds128(sa);
          bv4 = lds128(sa + SCB);
          ++sb;
        }
        constexpr int NW = KS * BITS / 32;  // words of the row (8 or 16)
        uint32_t wd[NW];
        const uint32_t wa = wr_a + uint32_t(slot * WSTG + row * (NW * 4));
#pragma unroll
        for (int h = 0; h < NW / 4; ++h) {
          const uint4 v = lds128(wa + uint32_t(16 * h));
          wd[4 * h] = v.x; wd[4 * h + 1] = v.y; wd[4 * h + 2] = v.z; wd[4 * h + 3] = v.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (g >= NA && ok)
          ok = mbar_wait(&aempty[ab], uint32_t(((g / NA) - 1) & 1), a.status, kErrWaitMma);
        tcg::tc_fence_after();
        const uint32_t s2 = dup_group(sv4, st & 7), b2 = dup_group(bv4, st & 7);
        uint32_t r[32];
        if (BITS == 4) {
          // word j holds k = 8j .. 8j+7 (nibble i at bits 4i): column 4j + c = pair (2c, 2c + 1)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t w = wd[j], u = w >> 4;
            const uint32_t c0 = __byte_perm(w, u, 0x0400u), c1 = __byte_perm(w, u, 0x0501u);
            const uint32_t c2 = __byte_perm(w, u, 0x0602u), c3 = __byte_perm(w, u, 0x0703u);
            r[4 * j + 0] = bf2_fma(bf2_sub(lop3_and_or(c0, 0x000F000Fu, M128), M128), s2, b2);
            r[4 * j + 1] = bf2_fma(bf2_sub(lop3_and_or(c1, 0x000F000Fu, M128), M128), s2, b2);
            r[4 * j + 2] = bf2_fma(bf2_sub(lop3_and_or(c2, 0x000F000Fu, M128), M128), s2, b2);
            r[4 * j + 3] = bf2_fma(bf2_sub(lop3_and_or(c3, 0x000F000Fu, M128), M128), s2, b2);
          }
        } else {
          // word j holds k = 4j .. 4j+3 (byte i): columns 2j (bytes 0, 1) and 2j + 1 (2, 3)
          constexpr uint32_t SIXTEEN = 0x41804180u;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const uint32_t w = wd[j], u = w >> 4;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const uint32_t sel = c ? 0x0302u : 0x0100u;
              const uint32_t lo = bf2_sub(lop3_and_or(__byte_perm(w, w, sel), 0x000F000Fu, M128), M128);
              const uint32_t hi = bf2_sub(lop3_and_or(__byte_perm(u, u, sel), 0x000F000Fu, M128), M128);
              r[2 * j + c] = bf2_fma(bf2_fma(hi, SIXTEEN, lo), s2, b2);
            }
          }
        }
        tcg::tmem_st32(ta + uint32_t(ab * 32), r);
        tcg::tmem_wait_st();
        tcg::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[ab]);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue: D -> bf16 y
    const int q = warp & 3, row = q * 32 + lane;
    int j = 0;
    for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x, ++j) {
      const int n = (t / a.ntm) * TN + row, m0 = (t % a.ntm) * TX;
      if (ok) ok = mbar_wait(dfull, uint32_t(j & 1), a.status, kErrWaitMma);
      tcg::tc_fence_after();
#pragma unroll 1
      for (int c0 = 0; c0 < TX; c0 += 32) {
        float v[32];
        tcg::tmem_ld32(tmem + (uint32_t(q * 32) << 16) + DCOL + uint32_t(c0), v);
        tcg::tmem_wait_ld();
        if (n < a.N) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int m = m0 + c0 + i;
            if (m < a.M) a.y[(size_t)m * a.ldy + n] = __float2bfloat16_rn(v[i]);
          }
        }
      }
      tcg::tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dempty);
    }
  }
  tcg::tc_fence_before();
  __syncthreads();
  tcg::tc_fence_after();
  if (warp == 0) tcg::tmem_dealloc(tmem, 512);
}

// x_n[m, k] = bf16(x[m, k] * rs[m] * w[k]) with rs[m] = rsqrt(sum_e ssq[e * stride + m] / K +
// eps): the RMSNorm prologue of the small-M engines (same statistics sum order, same rounding),
// applied once so that the wide kernel can read x by TMA. One CTA per row.
__global__ void __launch_bounds__(256) norm_apply_kernel(const bf16* x, long ldx, int K,
                                                         const bf16* w, const float* ssq,
                                                         int ssq_n, int ssq_stride, float eps,
                                                         bf16* xn, long ldn) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float rs;
  const int m = blockIdx.x;
  if (threadIdx.x < 32) {
    float ss = 0.f;
    for (int e = threadIdx.x; e < ssq_n; e += 32) ss += __ldcg(&ssq[(size_t)e * ssq_stride + m]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (threadIdx.x == 0) rs = rsqrtf(ss / float(K) + eps);
  }
  __syncthreads();
  const float r = rs;
  for (int c = threadIdx.x; c < K / 8; c += blockDim.x) {
    uint4 v = ldcg_v4(x + (size_t)m * ldx + c * 8);
    const uint4 wv = ldg_v4(w + c * 8);
    uint32_t* pv = reinterpret_cast<uint32_t*>(&v);
    const uint32_t* pw = reinterpret_cast<const uint32_t*>(&wv);
#pragma unroll
    for (int e = 0; e < 4; ++e)
      pv[e] = pack_bf16x2(bf16_lo(pv[e]) * r * bf16_lo(pw[e]), bf16_hi(pv[e]) * r * bf16_hi(pw[e]));
    *reinterpret_cast<uint4*>(xn + (size_t)m * ldn + c * 8) = v;
  }
}

// The fused epilogues on a bf16 product y: block (t, mb) loads rows mb*32 .. +31 of output tile
// t (128 columns) as fp32 and runs the same epilogue code as the small-M engines, which starts
// from the product rounded to bf16 — so the results equal the fused path's given equal products.
constexpr int EPSTR = 132;
template <int EPI>
__global__ void __launch_bounds__(128) epi_kernel(const QmmParams p, const bf16* y, long ldy) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[32 * EPSTR];
  const int t = blockIdx.x, mb = blockIdx.y * 32, n0 = t * 128;
  for (int idx = threadIdx.x; idx < 32 * 64; idx += blockDim.x) {
    const int r = idx >> 6, c2 = idx & 63;
    const int m = mb + r, n = n0 + 2 * c2;
    uint32_t v = 0u;
    if (m < p.M && n < p.N) v = __ldcg(reinterpret_cast<const unsigned int*>(y + (size_t)m * ldy + n));
    red[r * EPSTR + 2 * c2] = bf16_lo(v);
    red[r * EPSTR + 2 * c2 + 1] = bf16_hi(v);
  }
  __syncthreads();
  QmmParams q = p;
  q.M = min(32, p.M - mb);
  if (q.out) q.out += (size_t)mb * q.ldo;
  if (q.resid) q.resid += (size_t)mb * q.ldr;
  if (q.ssq_out) q.ssq_out += mb;
  if (q.qout) q.qout += (size_t)mb * q.ldq;
  if (q.row_pos) q.row_pos += mb;
  if (q.row_kv) q.row_kv += mb;
  epilogue<EPI, 128, EPSTR>(q, red, 0, 1, t, n0, 4, 0, nullptr);
}

}  // namespace wide

// ------------------------------------------------------------------------------ host side

template <int BITS>
static int launch_wide(const QmmParams& p, bf16* y, long ldy, cudaStream_t s) {
  constexpr wide::Layout L = wide::layout<BITS>();
  auto kern = wide::wide_kernel<BITS>;
  DSPARK_CUDA_TRY(configure_once(reinterpret_cast<const void*>(kern), 1, [&] {
                    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                L.total);
                  }),
                  "qmm_wide: set smem");
  CUtensorMap xmap, wmap, smap, bmap;
  const uint64_t words = (uint64_t)p.K * BITS / 32;
  const uint64_t G = (uint64_t)p.K / 64;
  if (!encode_tmap_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.x, p.K, p.M, (uint64_t)p.ldx * 2,
                      wide::KS, wide::TX, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.wq, words, p.N, words * 4,
                      wide::KS * BITS / 32, wide::TN, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_tmap_2d(&smap, CU_TENSOR_MAP_DATA_TYPE_UINT16, p.scales, G, p.N, G * 2, 8, wide::TN,
                      CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_tmap_2d(&bmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, p.biases, G, p.N, G * 2, 8, wide::TN,
                      CU_TENSOR_MAP_SWIZZLE_NONE))
    return DSPARK_ERR_CUDA;
  wide::WideArgs a;
  a.y = y;
  a.ldy = ldy;
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  a.ntm = (p.M + wide::TX - 1) / wide::TX;
  a.ntiles = a.ntm * ((p.N + wide::TN - 1) / wide::TN);
  a.status = p.status;
  const int grid = std::max(1, std::min(a.ntiles, sm_count(current_device())));
  DSPARK_CUDA_TRY(launch_ex(kern, dim3(grid), dim3(wide::NTHR), (size_t)L.total, s, 1, true,
                            xmap, wmap, smap, bmap, a),
                  "qmm_wide: launch");
  return DSPARK_OK;
}

int wide_product(const QmmParams& p, bf16* y, long ldy, cudaStream_t s) {
  if (p.bits != 4 && p.bits != 8) return fail(DSPARK_ERR_UNSUPPORTED, "qmm_wide: bits %d", p.bits);
  if (p.M < 1 || p.N < 1 || p.K < 64 || p.K % 64)
    return fail(DSPARK_ERR_UNSUPPORTED, "qmm_wide: M=%d N=%d K=%d (K %% 64 == 0)", p.M, p.N, p.K);
  if ((reinterpret_cast<uintptr_t>(p.x) & 15) || (p.ldx & 7) ||
      (reinterpret_cast<uintptr_t>(p.wq) & 15) || (reinterpret_cast<uintptr_t>(p.scales) & 15) ||
      (reinterpret_cast<uintptr_t>(p.biases) & 15) || (p.K / 64) % 8)
    return fail(DSPARK_ERR_UNSUPPORTED,
                "qmm_wide: x, weights, scales and biases must be 16-byte aligned, ldx %% 8 == 0 "
                "and K %% 512 == 0");
  if (y == nullptr) return fail(DSPARK_ERR_ARG, "qmm_wide: null output");
  return p.bits == 4 ? launch_wide<4>(p, y, ldy, s) : launch_wide<8>(p, y, ldy, s);
}

size_t wide_ws_bytes(int M, int K, int N, int epi, bool norm) {
  size_t b = 0;
  if (norm) b += ((size_t)M * K * 2 + 255) / 256 * 256;
  if (epi != EPI_PLAIN) b += ((size_t)M * N * 2 + 255) / 256 * 256;
  return b;
}

int run_wide(const QmmParams& p_in, int epi, void* ws, size_t ws_bytes, cudaStream_t s) {
  QmmParams p = p_in;
  if (p.status == nullptr) p.status = status_word(current_device());
  if (p.x_seg != 0 || p.ssq_seg != 0 || p.peer_world > 0 || p.wait_flag != nullptr)
    return fail(DSPARK_ERR_UNSUPPORTED, "qmm_wide: no segmented rows or peer transports");
  if (epi == EPI_PLAIN && p.bias != nullptr)
    return fail(DSPARK_ERR_UNSUPPORTED, "qmm_wide: no bias in the wide path");
  const bool norm = p.norm_w != nullptr;
  if (wide_ws_bytes(p.M, p.K, p.N, epi, norm) > ws_bytes || (ws == nullptr && (norm || epi != EPI_PLAIN)))
    return fail(DSPARK_ERR_ARG, "qmm_wide: needs %zu bytes of workspace (got %zu)",
                wide_ws_bytes(p.M, p.K, p.N, epi, norm), ws_bytes);
  char* w = static_cast<char*>(ws);
  if (norm) {
    bf16* xn = reinterpret_cast<bf16*>(w);
    w += ((size_t)p.M * p.K * 2 + 255) / 256 * 256;
    DSPARK_CUDA_TRY(launch_ex(wide::norm_apply_kernel, dim3(p.M), dim3(256), 0, s, 1, true, p.x,
                              p.ldx, p.K, p.norm_w, p.ssq_in, p.ssq_n, p.ssq_stride, p.eps, xn,
                              (long)p.K),
                    "qmm_wide: norm launch");
    p.x = xn;
    p.ldx = p.K;
  }
  if (epi == EPI_PLAIN) return wide_product(p, p.out, p.ldo, s);
  bf16* y = reinterpret_cast<bf16*>(w);
  const int rc = wide_product(p, y, p.N, s);
  if (rc != DSPARK_OK) return rc;
  const dim3 grid((p.N + 127) / 128, (p.M + 31) / 32);
  switch (epi) {
    case EPI_RESID:
      DSPARK_CUDA_TRY(launch_ex(wide::epi_kernel<EPI_RESID>, grid, dim3(128), 0, s, 1, true, p,
                                (const bf16*)y, (long)p.N), "qmm_wide: epilogue launch");
      break;
    case EPI_SWIGLU:
      DSPARK_CUDA_TRY(launch_ex(wide::epi_kernel<EPI_SWIGLU>, grid, dim3(128), 0, s, 1, true, p,
                                (const bf16*)y, (long)p.N), "qmm_wide: epilogue launch");
      break;
    case EPI_QKROPE:
      DSPARK_CUDA_TRY(launch_ex(wide::epi_kernel<EPI_QKROPE>, grid, dim3(128), 0, s, 1, true, p,
                                (const bf16*)y, (long)p.N), "qmm_wide: epilogue launch");
      break;
    default:
      return fail(DSPARK_ERR_ARG, "qmm_wide: bad epilogue %d", epi);
  }
  return DSPARK_OK;
}

}  // namespace qmm
}  // namespace dspark
