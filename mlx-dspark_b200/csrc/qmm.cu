// K1: small-M affine-quantized matmul  y[M,N] = x[M,K] . dequant(W)^T   (sm_100a)
//
// Replaces skinny_qmm.qmm (src/mlx_dspark/skinny_qmm.py:239-246, kernel :61-160) and the
// stock mx.quantized_matmul(transpose=True) it stands in for at 1-32 rows.
//
// Weight format (MLX affine, group 64): W packed as uint32 [N, K*bits/32], LSB-first; in
// 4-bit word j of a row holds k = 8j..8j+7 (k = 8j+s at bits 4s..4s+3), in 8-bit word j holds
// k = 4j..4j+3 (bits 8s..8s+7). scales/biases bf16 [N, K/64]; w = scale*q + bias.
//
// Design (B200-first, HBM-bound at these M):
//  * The packed weights stream through a ring of shared-memory stages filled by TMA
//    (cp.async.bulk.tensor, 128-byte swizzle, L2 evict-first) from one producer warp; the
//    scales/biases of each stage ride on the same mbarrier. The weight TMA of a launch is
//    issued before griddepcontrol.wait, so under programmatic dependent launch the weights
//    of layer i+1 stream while layer i finishes.
//  * Consumer warps dequantize in registers with the bf16 "magic exponent" trick: a nibble
//    OR'd into the mantissa of 128.0 is exactly 128+q (one lop3 per two weights); 8-bit
//    weights are split into low (128+lo) and high (2048+16*hi) nibble planes, two exact bf16
//    MMAs. The weights are the A operand of mma.m16n8k16 (16 output columns), the x rows the
//    B operand (8 rows per tile, M padded to 8/16/32), so a weight is read once per launch
//    whatever M is.
//  * Scale and bias factor out per group, as in the reference (skinny_qmm.py:131-145):
//    acc += scale*P + (bias - MAGIC*scale) * sum_k x, with P the exact per-group MMA sum.
//  * Split-K across the CTAs of a thread-block cluster; the fp32 partials are reduced in a
//    fixed rank order through distributed shared memory, so results are deterministic and
//    a row's output does not depend on M (the reference's row-count invariance,
//    tests/test_small_m_qmm.py:107-119).
//  * Epilogues: plain bf16 store (+ optional bias), residual add (+ per-row sum of squares
//    for the next RMSNorm), SwiGLU on interleaved gate/up rows, and Qwen3 q/k RMSNorm + RoPE
//    + KV-cache write. The prologue can apply RMSNorm to x while staging it.
#include <algorithm>
#include <cstdio>
#include <map>
#include <mutex>
#include <tuple>
#include <string>
#include <unordered_map>

#include "common.cuh"
#include "host_common.h"
#include "qmm.h"
#include "qmm_epilogue.cuh"

namespace dspark {
namespace qmm {

constexpr int KSTG = 512;        // k values per pipeline stage
constexpr int GPS = KSTG / 64;   // quantization groups per stage
constexpr int kSmemBudget = 220 * 1024;  // dynamic shared memory a plan may use at 32 rows

template <int BITS>
struct BitsTraits;
template <>
struct BitsTraits<4> {
  static constexpr float MAGIC = 128.0f;
  static constexpr int SB = 2;      // 128-byte TMA boxes per stage row (512 k * 4 bit)
  static constexpr int XPAD = 16;   // staged-x row padding (bytes)
};
template <>
struct BitsTraits<8> {
  static constexpr float MAGIC = 2176.0f;
  static constexpr int SB = 4;
  static constexpr int XPAD = 8;
};

// Physical tile row used by MMA row `gid` (0..7). Chosen so the warp's shared-memory loads
// of weight words are bank-conflict free under the 128-byte swizzle.
template <int BITS>
__device__ __forceinline__ int row_perm(int gid) {
  return BITS == 4 ? (((gid & 3) << 1) | (gid >> 2)) : (((gid & 1) << 2) | (gid >> 1));
}

struct SmemLayout {
  int ring, scs, bis, xs, sx, part, red, rs, bars, total;
};

template <int BITS, int NW, int RT>
__host__ __device__ inline SmemLayout smem_layout(int kslice, int nslots) {
  constexpr int TN = 16 * NW;
  constexpr int RP = 8 * RT;
  const int stg = BitsTraits<BITS>::SB * TN * 128;
  const int scb = TN * 16;
  SmemLayout L;
  int off = 0;
  L.ring = off;
  off += nslots * stg;
  L.scs = off;
  off += nslots * scb;
  L.bis = off;
  off += nslots * scb;
  L.xs = off;
  off += RP * (kslice * 2 + BitsTraits<BITS>::XPAD);
  off = (off + 15) & ~15;
  L.sx = off;
  off += RP * (kslice / 64) * 4;
  off = (off + 15) & ~15;
  L.part = off;
  off += RP * (TN + 4) * 4;
  L.red = off;
  off += RP * (TN + 4) * 4;
  L.rs = off;
  off += 32 * 4;
  off = (off + 15) & ~15;
  L.bars = off;
  off += 2 * nslots * 8;
  L.total = off + 1024;  // slack for aligning the dynamic base to 1024 bytes
  return L;
}

static int smem_bytes(int bits, int nw, int rt, int kslice, int nslots) {
  const int tn = 16 * nw, rp = 8 * rt;
  const int sb = bits == 4 ? BitsTraits<4>::SB : BitsTraits<8>::SB;
  const int xpad = bits == 4 ? BitsTraits<4>::XPAD : BitsTraits<8>::XPAD;
  int off = nslots * sb * tn * 128 + 2 * nslots * tn * 16;
  off += rp * (kslice * 2 + xpad);
  off = (off + 15) & ~15;
  off += rp * (kslice / 64) * 4;
  off = (off + 15) & ~15;
  off += 2 * rp * (tn + 4) * 4 + 32 * 4;
  off = (off + 15) & ~15;
  return off + 2 * nslots * 8 + 1024;
}

// ----------------------------------------------------------------------------- kernel

template <int BITS, int RT, int NW, int EPI, bool SCT>
__global__ void __launch_bounds__((NW + 1) * 32)
    qmm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
               const __grid_constant__ CUtensorMap bmap, const QmmParams p) {
  constexpr int TN = 16 * NW;
  constexpr int RP = 8 * RT;
  constexpr int NTHR = (NW + 1) * 32;
  constexpr int SB = BitsTraits<BITS>::SB;
  constexpr int BOX = TN * 128;
  constexpr int STG = SB * BOX;
  constexpr int SCB = TN * 16;
  constexpr float MAGIC = BitsTraits<BITS>::MAGIC;
  constexpr int PSTR = TN + 4;  // fp32 row stride of the partial / reduced tiles

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align_up<1024>(smem_raw);
  const int S = p.nslots;
  const SmemLayout Ls = smem_layout<BITS, NW, RT>(p.kslice, S);
  uint8_t* ring = smem + Ls.ring;
  uint8_t* scs = smem + Ls.scs;
  uint8_t* bis = smem + Ls.bis;
  uint8_t* xs = smem + Ls.xs;
  float* sx = reinterpret_cast<float*>(smem + Ls.sx);
  float* part = reinterpret_cast<float*>(smem + Ls.part);
  float* red = reinterpret_cast<float*>(smem + Ls.red);
  float* rsm = reinterpret_cast<float*>(smem + Ls.rs);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Ls.bars);
  uint64_t* empty = full + S;

  const int cs = p.cs;
  const int rank = blockIdx.x;  // cluster rank == split-K slice (cluster dims are (cs,1,1))
  const int ntile = blockIdx.y;
  const int n0 = ntile * TN;
  const int kbase = rank * p.kslice;
  const int kvalid = min(p.kslice, p.K - kbase);
  const int nst = (kvalid + KSTG - 1) / KSTG;
  const int gslice = p.kslice / 64;
  const int xrow = p.kslice * 2 + BitsTraits<BITS>::XPAD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == NW) {
    // ------------------------------------------------------------- producer warp
    if (lane == 0) {
      prefetch_tmap(&wmap);
      if (SCT) {
        prefetch_tmap(&smap);
        prefetch_tmap(&bmap);
      }
      const uint64_t pol = l2_policy_evict_first();
      const uint32_t bytes = STG + (SCT ? 2 * SCB : 0);
      for (int st = 0; st < nst; ++st) {
        const int slot = st % S;
        if (st >= S) {
          if (!mbar_wait(&empty[slot], ((st / S) - 1) & 1, p.status, kErrWaitEmpty)) break;
        }
        mbar_arrive_expect_tx(&full[slot], bytes);
        const int kk = kbase + st * KSTG;
        const int w0 = kk * BITS / 32;
#pragma unroll
        for (int b = 0; b < SB; ++b)
          tma_load_2d(ring + slot * STG + b * BOX, &wmap, &full[slot], w0 + b * 32, n0, pol);
        if (SCT) {
          tma_load_2d(scs + slot * SCB, &smap, &full[slot], kk / 64, n0, pol);
          tma_load_2d(bis + slot * SCB, &bmap, &full[slot], kk / 64, n0, pol);
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------- consumer warps
    pdl_wait();  // x / residual / norm statistics come from earlier kernels
    constexpr int NC = NW * 32;
    const int tid = threadIdx.x;

    // RMSNorm statistics for the prologue: rs[m] = 1/sqrt(mean(x^2) + eps)
    if (p.norm_w != nullptr) {
      // one warp per row: lanes stride over the partial sums (fixed order per lane, then a
      // fixed shuffle tree: deterministic)
      for (int m = warp; m < RP; m += NW) {
        float ss = 0.f;
        if (m < p.M)
          for (int e = lane; e < p.ssq_n; e += 32) ss += __ldcg(&p.ssq_in[e * p.ssq_stride + m]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) rsm[m] = m < p.M ? rsqrtf(ss / float(p.K) + p.eps) : 0.f;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(NC));
    }

    // Stage x[:, kbase : kbase + kslice] into shared memory in MMA-operand order. Each thread
    // issues XB 16-byte loads before using any, so the staging costs ~one L2 round trip per
    // batch instead of one per block. x is read through L2 only (ld.global.cg): it was
    // written by the previous kernel.
    const int blocks = p.kslice / 8;
    const int total = RP * blocks;
    constexpr int XB = 8;
    const bool nrm = p.norm_w != nullptr;
    for (int base = tid; base < total; base += NC * XB) {
      uint4 v[XB], w[XB];
#pragma unroll
      for (int u = 0; u < XB; ++u) {
        const int idx = base + u * NC;
        const int m = idx / blocks, j = idx - m * blocks;
        v[u] = make_uint4(0u, 0u, 0u, 0u);
        w[u] = v[u];
        if (idx < total && m < p.M && j * 8 < kvalid) {
          const int k = kbase + j * 8;
          v[u] = __ldcg(reinterpret_cast<const uint4*>(p.x + (size_t)m * p.ldx + k));
          if (nrm) w[u] = __ldg(reinterpret_cast<const uint4*>(p.norm_w + k));
        }
      }
#pragma unroll
      for (int u = 0; u < XB; ++u) {
        const int idx = base + u * NC;
        if (idx >= total) break;
        const int m = idx / blocks, j = idx - m * blocks;
        uint4 vv = v[u];
        if (nrm && m < p.M) {
          const float r = rsm[m];
          uint32_t* pv = reinterpret_cast<uint32_t*>(&vv);
          const uint32_t* pw = reinterpret_cast<const uint32_t*>(&w[u]);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            pv[e] = pack_bf16x2(bf16_lo(pv[e]) * r * bf16_lo(pw[e]),
                                bf16_hi(pv[e]) * r * bf16_hi(pw[e]));
        }
        uint8_t* dst = xs + m * xrow + j * 16;
        if (BITS == 4) {  // 8-block order (0,4,1,5,2,6,3,7)
          uint4 o;
          o.x = __byte_perm(vv.x, vv.z, 0x5410);
          o.y = __byte_perm(vv.x, vv.z, 0x7632);
          o.z = __byte_perm(vv.y, vv.w, 0x5410);
          o.w = __byte_perm(vv.y, vv.w, 0x7632);
          *reinterpret_cast<uint4*>(dst) = o;
        } else {          // two 4-blocks, each in order (0,2,1,3)
          uint2 a, b;
          a.x = __byte_perm(vv.x, vv.y, 0x5410);
          a.y = __byte_perm(vv.x, vv.y, 0x7632);
          b.x = __byte_perm(vv.z, vv.w, 0x5410);
          b.y = __byte_perm(vv.z, vv.w, 0x7632);
          reinterpret_cast<uint2*>(dst)[0] = a;
          reinterpret_cast<uint2*>(dst)[1] = b;
        }
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(NC));
    // Per-group input sums (fixed order: deterministic, row-local), stored group-major.
    for (int idx = tid; idx < RP * gslice; idx += NC) {
      const int g = idx / RP, m = idx - g * RP;  // rows fastest: conflict-free 16-byte loads
      const uint8_t* src = xs + m * xrow + g * 128;
      float s = 0.f;
      if (BITS == 4) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint4 q = *reinterpret_cast<const uint4*>(src + 16 * i);
          s += (bf16_lo(q.x) + bf16_hi(q.x)) + (bf16_lo(q.y) + bf16_hi(q.y)) +
               (bf16_lo(q.z) + bf16_hi(q.z)) + (bf16_lo(q.w) + bf16_hi(q.w));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint2 q = *reinterpret_cast<const uint2*>(src + 8 * i);
          s += (bf16_lo(q.x) + bf16_hi(q.x)) + (bf16_lo(q.y) + bf16_hi(q.y));
        }
      }
      sx[g * RP + m] = s;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(NC));

    const int gid = lane >> 2, tig = lane & 3;
    const int ra = warp * 16 + row_perm<BITS>(gid);
    const int rb = ra + 8;
    float acc[RT][4];
#pragma unroll
    for (int r = 0; r < RT; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[r][c] = 0.f;

    const uint32_t ring_a = smem_u32(ring);
    const uint32_t xs_a = smem_u32(xs);
    const int gfirst = kbase / 64;

    for (int st = 0; st < nst; ++st) {
      const int slot = st % S;
      mbar_wait(&full[slot], (st / S) & 1, p.status, kErrWaitFull);
      const uint32_t wbase = ring_a + slot * STG;
      uint4 sca, scb_, bia, bib;
      if (SCT) {
        sca = lds128(smem_u32(scs + slot * SCB + ra * 16));
        scb_ = lds128(smem_u32(scs + slot * SCB + rb * 16));
        bia = lds128(smem_u32(bis + slot * SCB + ra * 16));
        bib = lds128(smem_u32(bis + slot * SCB + rb * 16));
      }
#pragma unroll
      for (int gi = 0; gi < GPS; ++gi) {
        const int gl = st * GPS + gi;  // group index within this slice
        if (gfirst + gl >= p.G || gl * 64 >= kvalid) break;
        float P[RT][4];
#pragma unroll
        for (int r = 0; r < RT; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c) P[r][c] = 0.f;

        if (BITS == 4) {
          // words gi*8 + 2*tig + {0,1} of rows ra / rb
          const int box = gi >> 2;
          const int chunk = ((gi & 3) << 1) + (tig >> 1);
          const int within = (tig & 1) * 8;
          const uint2 wa = lds64(wbase + box * BOX + ra * 128 + ((chunk ^ (ra & 7)) << 4) + within);
          const uint2 wb = lds64(wbase + box * BOX + rb * 128 + ((chunk ^ (rb & 7)) << 4) + within);
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const uint32_t xa = h2 ? wa.y : wa.x;
            const uint32_t xb = h2 ? wb.y : wb.x;
            uint32_t A[4], Bq[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              A[i] = lop3_and_or(xa >> (4 * i), 0x000F000Fu, 0x43004300u);
              Bq[i] = lop3_and_or(xb >> (4 * i), 0x000F000Fu, 0x43004300u);
            }
            const int blk = st * 64 + gi * 8 + 2 * tig + h2;  // 8-k block within the slice
#pragma unroll
            for (int r = 0; r < RT; ++r) {
              const uint4 xv = lds128(xs_a + (r * 8 + gid) * xrow + blk * 16);
              mma_bf16_16816(P[r], A[0], Bq[0], A[1], Bq[1], xv.x, xv.y);
              mma_bf16_16816(P[r], A[2], Bq[2], A[3], Bq[3], xv.z, xv.w);
            }
          }
        } else {
          // words gi*16 + 4*tig + {0..3} of rows ra / rb
          const int box = gi >> 1;
          const int chunk = ((gi & 1) << 2) + tig;
          const uint4 wa = lds128(wbase + box * BOX + ra * 128 + ((chunk ^ (ra & 7)) << 4));
          const uint4 wb = lds128(wbase + box * BOX + rb * 128 + ((chunk ^ (rb & 7)) << 4));
          const uint32_t wav[4] = {wa.x, wa.y, wa.z, wa.w};
          const uint32_t wbv[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const uint32_t xa = wav[h], xb = wbv[h];
            const uint32_t alo0 = lop3_and_or(xa, 0x000F000Fu, 0x43004300u);
            const uint32_t alo1 = lop3_and_or(xa >> 8, 0x000F000Fu, 0x43004300u);
            const uint32_t ahi0 = lop3_and_or(xa >> 4, 0x000F000Fu, 0x45004500u);
            const uint32_t ahi1 = lop3_and_or(xa >> 12, 0x000F000Fu, 0x45004500u);
            const uint32_t blo0 = lop3_and_or(xb, 0x000F000Fu, 0x43004300u);
            const uint32_t blo1 = lop3_and_or(xb >> 8, 0x000F000Fu, 0x43004300u);
            const uint32_t bhi0 = lop3_and_or(xb >> 4, 0x000F000Fu, 0x45004500u);
            const uint32_t bhi1 = lop3_and_or(xb >> 12, 0x000F000Fu, 0x45004500u);
            const int kq = st * KSTG + (gi * 16 + 4 * tig + h) * 4;  // k within slice
#pragma unroll
            for (int r = 0; r < RT; ++r) {
              const uint2 xv = lds64(xs_a + (r * 8 + gid) * xrow + kq * 2);
              mma_bf16_16816(P[r], alo0, blo0, alo1, blo1, xv.x, xv.y);
              mma_bf16_16816(P[r], ahi0, bhi0, ahi1, bhi1, xv.x, xv.y);
            }
          }
        }
        // fold the group: acc += s*P + (b - MAGIC*s) * sum(x)
        float sa, sbv, ba, bb;
        if (SCT) {
          const uint32_t* pa = reinterpret_cast<const uint32_t*>(&sca);
          const uint32_t* pb = reinterpret_cast<const uint32_t*>(&scb_);
          const uint32_t* qa = reinterpret_cast<const uint32_t*>(&bia);
          const uint32_t* qb = reinterpret_cast<const uint32_t*>(&bib);
          sa = (gi & 1) ? bf16_hi(pa[gi >> 1]) : bf16_lo(pa[gi >> 1]);
          sbv = (gi & 1) ? bf16_hi(pb[gi >> 1]) : bf16_lo(pb[gi >> 1]);
          ba = (gi & 1) ? bf16_hi(qa[gi >> 1]) : bf16_lo(qa[gi >> 1]);
          bb = (gi & 1) ? bf16_hi(qb[gi >> 1]) : bf16_lo(qb[gi >> 1]);
        } else {
          const int g = gfirst + gl;
          const int na = min(n0 + ra, p.N - 1), nb = min(n0 + rb, p.N - 1);
          sa = bf2f(p.scales[(size_t)na * p.G + g]);
          sbv = bf2f(p.scales[(size_t)nb * p.G + g]);
          ba = bf2f(p.biases[(size_t)na * p.G + g]);
          bb = bf2f(p.biases[(size_t)nb * p.G + g]);
        }
        const float ca = ba - MAGIC * sa, cb = bb - MAGIC * sbv;
#pragma unroll
        for (int r = 0; r < RT; ++r) {
          const float2 s2 = *reinterpret_cast<const float2*>(&sx[gl * RP + r * 8 + 2 * tig]);
          acc[r][0] = fmaf(sa, P[r][0], fmaf(ca, s2.x, acc[r][0]));
          acc[r][1] = fmaf(sa, P[r][1], fmaf(ca, s2.y, acc[r][1]));
          acc[r][2] = fmaf(sbv, P[r][2], fmaf(cb, s2.x, acc[r][2]));
          acc[r][3] = fmaf(sbv, P[r][3], fmaf(cb, s2.y, acc[r][3]));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }

    // partial tile -> shared memory [m][n]
#pragma unroll
    for (int r = 0; r < RT; ++r) {
      const int m = r * 8 + 2 * tig;
      part[m * PSTR + ra] = acc[r][0];
      part[(m + 1) * PSTR + ra] = acc[r][1];
      part[m * PSTR + rb] = acc[r][2];
      part[(m + 1) * PSTR + rb] = acc[r][3];
    }
    __syncwarp();
  }

  // ------------------------------------------------------------- split-K reduction
  if (cs > 1) cluster_sync_all(); else __syncthreads();
  const int nmine = (p.M > rank) ? (p.M - rank + cs - 1) / cs : 0;  // rows m = rank + i*cs
  for (int idx = threadIdx.x; idx < nmine * (TN / 4); idx += NTHR) {
    const int mi = idx / (TN / 4), n4 = idx - mi * (TN / 4);
    const int m = rank + mi * cs;
    const uint32_t a = smem_u32(&part[m * PSTR + n4 * 4]);
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    if (cs > 1) {
      for (int c = 0; c < cs; ++c) {
        const float4 v = ld_dsmem_f4(mapa_shared(a, c));
        s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
      }
    } else {
      s = *reinterpret_cast<const float4*>(&part[m * PSTR + n4 * 4]);
    }
    *reinterpret_cast<float4*>(&red[m * PSTR + n4 * 4]) = s;
  }
  if (cs > 1) cluster_sync_all(); else __syncthreads();

  epilogue<EPI, TN, PSTR>(p, red, rank, cs, ntile, n0, NW + 1);
}

// ----------------------------------------------------------------------------- host side

struct TmapKey {
  const void* ptr;
  uint64_t d0, d1, stride;
  uint32_t b0, b1;
  int dt, swz;
  bool operator==(const TmapKey& o) const {
    return ptr == o.ptr && d0 == o.d0 && d1 == o.d1 && stride == o.stride && b0 == o.b0 &&
           b1 == o.b1 && dt == o.dt && swz == o.swz;
  }
};
struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    size_t h = reinterpret_cast<size_t>(k.ptr);
    h ^= (k.d0 * 0x9E3779B97F4A7C15ull) ^ (k.d1 << 17) ^ (k.stride << 5) ^ (size_t(k.b1) << 40);
    return h;
  }
};

static std::mutex g_tmap_mu;
static std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> g_tmap_cache;

static bool get_tmap(CUtensorMap* out, CUtensorMapDataType dt, const void* base, uint64_t d0,
                     uint64_t d1, uint64_t stride, uint32_t b0, uint32_t b1,
                     CUtensorMapSwizzle swz) {
  TmapKey key{base, d0, d1, stride, b0, b1, int(dt), int(swz)};
  {
    std::lock_guard<std::mutex> lk(g_tmap_mu);
    auto it = g_tmap_cache.find(key);
    if (it != g_tmap_cache.end()) {
      *out = it->second;
      return true;
    }
  }
  if (!encode_tmap_2d(out, dt, base, d0, d1, stride, b0, b1, swz)) return false;
  std::lock_guard<std::mutex> lk(g_tmap_mu);
  if (g_tmap_cache.size() > 65536) g_tmap_cache.clear();
  g_tmap_cache[key] = *out;
  return true;
}

bool tma_maps(const QmmParams& p, int tn, bool sct, CUtensorMap* wmap, CUtensorMap* smap,
              CUtensorMap* bmap) {
  const uint64_t words = (uint64_t)p.K * p.bits / 32;
  if (!get_tmap(wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.wq, words, p.N, words * 4, 32, tn,
                CU_TENSOR_MAP_SWIZZLE_128B))
    return false;
  if (sct) {
    if (!get_tmap(smap, CU_TENSOR_MAP_DATA_TYPE_UINT16, p.scales, p.G, p.N, (uint64_t)p.G * 2, 8,
                  tn, CU_TENSOR_MAP_SWIZZLE_NONE))
      return false;
    if (!get_tmap(bmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, p.biases, p.G, p.N, (uint64_t)p.G * 2, 8,
                  tn, CU_TENSOR_MAP_SWIZZLE_NONE))
      return false;
  } else {
    *smap = *wmap;
    *bmap = *wmap;
  }
  return true;
}

template <int BITS, int RT, int NW, int EPI, bool SCT>
static int launch_one(const QmmParams& p, const QmmPlan& pl, cudaStream_t stream) {
  auto kern = qmm_kernel<BITS, RT, NW, EPI, SCT>;
  constexpr int TN = 16 * NW;
  const SmemLayout L = smem_layout<BITS, NW, RT>(pl.kslice, pl.nslots);
  // configured per device with the largest dynamic shared memory asked for so far
  DSPARK_CUDA_TRY(configure_once(reinterpret_cast<const void*>(kern), L.total, [&] {
                    cudaError_t e = cudaFuncSetAttribute(
                        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total);
                    if (e == cudaSuccess)
                      e = cudaFuncSetAttribute(
                          kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
                    const int carve = env_int("DSPARK_QMM_CARVEOUT", -1);
                    if (e == cudaSuccess && carve >= 0)
                      e = cudaFuncSetAttribute(
                          kern, cudaFuncAttributePreferredSharedMemoryCarveout, carve);
                    return e;
                  }),
                  "qmm: set smem / cluster attributes");
  CUtensorMap wmap, smap, bmap;
  if (!tma_maps(p, TN, SCT, &wmap, &smap, &bmap)) return DSPARK_ERR_CUDA;
  dim3 grid(pl.cs, (p.N + TN - 1) / TN);
  dim3 block((NW + 1) * 32);
  DSPARK_CUDA_TRY(launch_ex(kern, grid, block, (size_t)L.total, stream, pl.cs, true, wmap, smap, bmap, p),
                  "qmm: launch");
  return DSPARK_OK;
}

template <int BITS, int RT, int EPI>
static int dispatch_nw(const QmmParams& p, const QmmPlan& pl, cudaStream_t s) {
  const bool sct = pl.sct;
  if constexpr (EPI == EPI_PLAIN) {
    if (pl.nw == 2) return sct ? launch_one<BITS, RT, 2, EPI, true>(p, pl, s) : launch_one<BITS, RT, 2, EPI, false>(p, pl, s);
    if (pl.nw == 4) return sct ? launch_one<BITS, RT, 4, EPI, true>(p, pl, s) : launch_one<BITS, RT, 4, EPI, false>(p, pl, s);
    if (pl.nw == 8) return sct ? launch_one<BITS, RT, 8, EPI, true>(p, pl, s) : launch_one<BITS, RT, 8, EPI, false>(p, pl, s);
  } else if constexpr (EPI == EPI_QKROPE) {
    if (!sct) return fail(DSPARK_ERR_UNSUPPORTED, "qmm: fused epilogues need K %% 512 == 0");
    if (pl.nw == 8) return launch_one<BITS, RT, 8, EPI, true>(p, pl, s);
  } else {
    if (!sct) return fail(DSPARK_ERR_UNSUPPORTED, "qmm: fused epilogues need K %% 512 == 0");
    if (pl.nw == 4) return launch_one<BITS, RT, 4, EPI, true>(p, pl, s);
    if (pl.nw == 8) return launch_one<BITS, RT, 8, EPI, true>(p, pl, s);
  }
  return fail(DSPARK_ERR_UNSUPPORTED, "qmm: no kernel for %d warps with epilogue %d", pl.nw, EPI);
}

template <int BITS, int EPI>
static int dispatch_rt(const QmmParams& p, const QmmPlan& pl, cudaStream_t s) {
  if (p.M <= 8) return dispatch_nw<BITS, 1, EPI>(p, pl, s);
  if (p.M <= 16) return dispatch_nw<BITS, 2, EPI>(p, pl, s);
  return dispatch_nw<BITS, 4, EPI>(p, pl, s);
}

// Launch geometry for [N, K] at `bits` and row class rt: tile width (16 * nw output
// columns), split-K factor (cluster size) and ring depth. Modelled per SM as: the bytes its
// CTAs stream (load balance over SMs), a fixed per-CTA latency (x staging, first TMA bytes,
// split-K reduction), and a penalty for shallow pipelines.
static QmmPlan plan_mma(int N, int K, int bits, int epi, int min_tn, int rt);

// Engine choice: DSPARK_QMM_IMPL = "st" (default: streaming), "tc" (tcgen05 / TMEM) or "mma"
// (per-tile CTAs). Shapes an engine cannot serve fall through to the next one.
static int impl_choice() {
  const char* v = std::getenv("DSPARK_QMM_IMPL");
  if (v == nullptr) return 2;
  const std::string s(v);
  return s == "mma" ? 0 : s == "tc" ? 1 : 2;
}

QmmPlan plan(int N, int K, int bits, int epi, int min_tn, int rt) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int, int, int>, QmmPlan> cache;
  const int impl = impl_choice();
  const auto key = std::make_tuple(current_device(), N, K, bits, epi * 64 + min_tn, rt, impl);
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  QmmPlan pl;
  pl.nw = 0;
  if (impl == 2) pl = plan_st(N, K, bits, rt);
  if (impl == 2 && rt == 4 && pl.nw != 0 && !pl.tcmma) {
    // the 16-row plan twice, when the model prefers it (rows 0-15 and the rest)
    const QmmPlan h = plan_st(N, K, bits, 2);
    if (h.nw != 0 && !h.tcmma && 2.0 * h.model_s < pl.model_s) pl.halves = true;
  }
  if (pl.nw == 0 && impl >= 1) pl = plan_tc(N, K, bits, rt);
  // shapes whose x slice and ring fit neither persistent engine run on per-tile CTAs (the same
  // contract, all hand-written CUDA)
  if (pl.nw == 0) pl = plan_mma(N, K, bits, epi, min_tn, rt);
  std::lock_guard<std::mutex> g(mu);
  cache[key] = pl;
  return pl;
}

// Streaming engine: choose the split-K factor cs (= cluster size), the ring depth and the
// number of persistent clusters. Modelled as: every cluster walks ceil(tiles / clusters) tiles,
// each CTA streaming 128 rows x K/cs of weights (+ scales/biases) at the smaller of a per-CTA
// consumer rate and its share of HBM bandwidth, plus a per-tile cost (split-K exchange,
// epilogue) and the x staging of its K slice, which grows with the rows staged.
// The terms are a least-squares fit to B200 sweeps of every split over the Qwen3-8B
// projections (4-bit, 1 and 16 rows): per streamed KB 0.015 + 0.013 * mt us (mt = 8-row
// column tiles), 0.5 us per tile, 0.29 * mt us per 1024 k staged. The fit picks the fastest
// measured split for all four shapes at 16 rows. DSPARK_QMM_PLAN_LOG=1 prints every candidate.
QmmPlan plan_st(int N, int K, int bits, int rt) {
  QmmPlan pl;
  pl.engine = 2;
  pl.nw = 0;
  pl.rt = rt;
  pl.sct = true;
  if (K % 512) return pl;
  const int force_cs = env_int("DSPARK_QMM_CS", 0);
  const int max_slots = std::max(3, env_int("DSPARK_QMM_SLOTS", 8));
  const int force_clusters = env_int("DSPARK_QMM_CLUSTERS", 0);
  pl.tcmma = env_int("DSPARK_QMM_ST_TC", 0) != 0;  // tcgen05 consumers measured slower
  const double hbm = env_int("DSPARK_QMM_HBM_GBS", 6500) * 1e9;
  const int mt = rt <= 1 ? 1 : rt <= 2 ? 2 : 4;
  // bytes/s one CTA's consumers take in; 8-bit weights carry half the MACs per byte
  const double cta_rate = 1e3 / ((0.015 + 0.013 * mt) * 1e-6) * (bits == 8 ? 1.5 : 1.0);
  const int sm_mbs = env_int("DSPARK_QMM_SM_MBS", 0);
  const double sm_cap = sm_mbs > 0 ? sm_mbs * 1e6 : cta_rate;
  const double t_tile = env_int("DSPARK_QMM_TILE_NS", 500) * 1e-9;
  const bool log = env_int("DSPARK_QMM_PLAN_LOG", 0) != 0;
  const int ntiles = (N + 127) / 128;
  double best = 1e30;
  for (int cs : {1, 2, 3, 4, 5, 6, 8, 10, 12, 16}) {
    if (force_cs && cs != force_cs) continue;
    const int kslice = ((K + cs - 1) / cs + 511) / 512 * 512;
    if ((cs - 1) * kslice >= K) continue;
    if (kslice > 8192) continue;  // x is staged in at most 16 blocks of 512 k
    int slots = max_slots;
    while (slots >= 3 && st_smem_bytes(bits, mt, kslice, slots, cs, pl.tcmma) > 227 * 1024) --slots;
    if (slots < 3) continue;
    const int smem = st_smem_bytes(bits, mt, kslice, slots, cs, pl.tcmma);
    int clusters = std::min(ntiles, st_max_clusters(cs, smem));
    if (force_clusters > 0) clusters = std::min(ntiles, force_clusters);
    if (clusters < 1) continue;
    const int waves = (ntiles + clusters - 1) / clusters;
    const double tile_bytes = 128.0 * kslice * (bits / 8.0 + 4.0 / 64.0);
    const double rate = std::min(sm_cap, hbm / (clusters * cs));
    double t = waves * (tile_bytes / rate + t_tile) + 1.5e-6 + 0.29e-6 * mt * kslice / 1024.0;
    if (cs & (cs - 1)) t *= 1.03;  // odd cluster shapes pack less evenly into GPCs
    if (log)
      std::fprintf(stderr,
                   "plan_st N=%d K=%d bits=%d rt=%d cs=%d kslice=%d slots=%d clusters=%d waves=%d "
                   "model_us=%.3f\n",
                   N, K, bits, rt, cs, kslice, slots, clusters, waves, t * 1e6);
    if (t < best) {
      best = t;
      pl.nw = 8;  // 128-row tile
      pl.cs = cs;
      pl.kslice = kslice;
      pl.nslots = slots;
      pl.clusters = clusters;
      pl.model_s = t;
    }
  }
  return pl;
}

// tcgen05 engine (persistent clusters): choose the split-K factor cs (= cluster size), the ring
// depth and the number of clusters. Modelled as: every cluster walks ceil(tiles / clusters)
// tiles, each CTA streaming 128 rows x K/cs of weights (+ scales/biases) at the smaller of a
// per-SM streaming cap and its share of HBM bandwidth, plus a once-per-CTA start (x staging,
// ring fill) and a small per-tile cost (split-K exchange, epilogue).
QmmPlan plan_tc(int N, int K, int bits, int rt) {
  QmmPlan pl;
  pl.engine = 1;
  pl.nw = 0;
  pl.rt = rt;
  pl.sct = (K % 512 == 0);
  const int force_cs = env_int("DSPARK_QMM_CS", 0);
  const int max_slots = std::max(2, env_int("DSPARK_QMM_SLOTS", 8));
  const int force_clusters = env_int("DSPARK_QMM_CLUSTERS", 0);
  // measured on B200 (4-bit, 16 rows): one CTA streams ~16.5 GB/s through dequant + MMA + fold,
  // and a tile costs ~2.2 us more (split-K exchange, epilogue, pipeline turn-around)
  const double hbm = 6.5e12, sm_cap = 1.65e10 * (bits == 8 ? 2.0 : 1.0), t_tile = 2.2e-6;
  const int ntiles = (N + 127) / 128;
  double best = 1e30;
  for (int cs : {1, 2, 3, 4, 5, 6, 8, 10, 12, 16}) {
    if (force_cs && cs != force_cs) continue;
    const int kslice = ((K + cs - 1) / cs + KSTG - 1) / KSTG * KSTG;
    if ((cs - 1) * kslice >= K) continue;
    // the split depends on the shape and the row class only, so within a class a row's result
    // never depends on how many rows ride with it
    const int slots = std::min(max_slots, (kSmemBudget - tc_smem_bytes(bits, rt, kslice, 0)) /
                                              tc_stage_bytes(bits));
    if (slots < 2) continue;
    const int smem = tc_planned_smem(bits, rt, kslice, slots);
    int clusters = std::min(ntiles, tc_max_clusters(bits, rt, cs, smem));
    if (force_clusters > 0) clusters = std::min(ntiles, force_clusters);
    if (clusters < 1) continue;
    const int waves = (ntiles + clusters - 1) / clusters;
    const double tile_bytes = 128.0 * kslice * (bits / 8.0 + 4.0 / 64.0);
    const double rate = std::min(sm_cap, hbm / (clusters * cs));
    double t = waves * (tile_bytes / rate + t_tile) + 1.5e-6 + kslice * 32.0 / 2e11;
    if (slots < 3) t *= 1.15;
    if (cs & (cs - 1)) t *= 1.05;  // odd cluster shapes pack less evenly into GPCs
    if (t < best) {
      best = t;
      pl.nw = 8;  // 128-row tile
      pl.cs = cs;
      pl.kslice = kslice;
      pl.nslots = slots;
      pl.clusters = clusters;
    }
  }
  return pl;
}

static QmmPlan plan_mma(int N, int K, int bits, int epi, int min_tn, int rt) {
  QmmPlan pl;
  pl.engine = 0;
  const int sms = sm_count(current_device());
  pl.sct = (K % 512 == 0);
  int nw_choices[3] = {2, 4, 8};
  double best = 1e30;
  const int force_nw = env_int("DSPARK_QMM_NW", 0);
  const int force_cs = env_int("DSPARK_QMM_CS", 0);
  const double bw_sm = 6.5e12 / sms;     // bytes/s each SM can draw when all stream
  const double t_fix = 2.0e-6;           // per-CTA fixed latency (s)
  for (int nw : nw_choices) {
    if (16 * nw < min_tn) continue;
    if (epi != EPI_PLAIN && nw == 2) continue;
    if (epi == EPI_QKROPE && nw != 8) continue;
    if (force_nw && nw != force_nw) continue;
    const int tn = 16 * nw;
    const int ntiles = (N + tn - 1) / tn;
    for (int cs = 1; cs <= 16; ++cs) {
      if (force_cs && cs != force_cs) continue;
      if (cs > 8 && cs != 16) continue;
      const int kslice = ((K + cs - 1) / cs + KSTG - 1) / KSTG * KSTG;
      if ((cs - 1) * kslice >= K) continue;  // every rank needs work
      const int nst = (kslice + KSTG - 1) / KSTG;
      const int ctas = cs * ntiles;
      const double wbytes = double(tn) * kslice * bits / 8.0;  // weight bytes per CTA
      int slots = std::min(nst, std::max(1, env_int("DSPARK_QMM_SLOTS", 4)));
      while (slots > 1 && smem_bytes(bits, nw, rt, kslice, slots) > kSmemBudget) --slots;
      if (smem_bytes(bits, nw, rt, kslice, slots) > kSmemBudget) continue;
      const int smem = smem_bytes(bits, nw, rt, kslice, slots);
      const int occ = std::max(1, std::min(2048 / (32 * (nw + 1)), (227 * 1024) / std::max(smem, 1)));
      // CTAs per SM over the launch, and the SM that gets the most
      const double per_sm = std::ceil(double(ctas) / sms);
      const double rounds = std::ceil(per_sm / occ);
      double t = per_sm * wbytes / bw_sm + rounds * t_fix;
      if (slots < std::min(nst, 3)) t *= 1.0 + 0.25 * (std::min(nst, 3) - slots);
      t *= 1.0 + 0.01 * (cs - 1);  // split-K reduction
      if (t < best) {
        best = t;
        pl.nw = nw;
        pl.cs = cs;
        pl.kslice = kslice;
        pl.nslots = slots;
      }
    }
  }
  if (best >= 1e30) pl.nw = 0;
  pl.rt = rt;
  return pl;
}

int run(const QmmParams& p_in, int epi, const QmmPlan* plan_in, cudaStream_t stream) {
  QmmParams p = p_in;
  if (p.bits != 4 && p.bits != 8) return fail(DSPARK_ERR_UNSUPPORTED, "qmm: bits must be 4 or 8 (got %d)", p.bits);
  if (p.M < 1 || p.M > 32) return fail(DSPARK_ERR_UNSUPPORTED, "qmm: M=%d outside 1..32", p.M);
  if (p.K <= 0 || p.K % 64 || p.N <= 0 || p.N % 8)
    return fail(DSPARK_ERR_UNSUPPORTED, "qmm: need K %% 64 == 0 and N %% 8 == 0 (K=%d N=%d)", p.K, p.N);
  if ((reinterpret_cast<uintptr_t>(p.x) & 15) || (p.ldx & 7))
    return fail(DSPARK_ERR_UNSUPPORTED, "qmm: x must be 16-byte aligned with ldx %% 8 == 0");
  if ((reinterpret_cast<uintptr_t>(p.wq) & 15) || (reinterpret_cast<uintptr_t>(p.out) & 3) || (p.ldo & 1))
    return fail(DSPARK_ERR_UNSUPPORTED, "qmm: weights must be 16-byte aligned, out 4-byte aligned with even ldo");
  if ((reinterpret_cast<uintptr_t>(p.norm_w) & 15) || (p.resid && ((reinterpret_cast<uintptr_t>(p.resid) & 3) || (p.ldr & 1))))
    return fail(DSPARK_ERR_UNSUPPORTED, "qmm: norm weight must be 16-byte aligned, residual 4-byte aligned");
  p.G = p.K / 64;
  if (p.status == nullptr) p.status = status_word(current_device());
  const int rt = p.M <= 16 ? 2 : 4;
  QmmPlan pl = plan_in ? *plan_in : plan(p.N, p.K, p.bits, epi, epi == EPI_QKROPE ? 128 : 0, rt);
  if (pl.nw == 0) return fail(DSPARK_ERR_UNSUPPORTED, "qmm: no launch geometry for N=%d K=%d", p.N, p.K);
  if (pl.rt < rt)
    return fail(DSPARK_ERR_ARG, "qmm: plan made for %d rows used for M=%d", 8 * pl.rt, p.M);
  if (pl.sct && ((reinterpret_cast<uintptr_t>(p.scales) & 15) || (reinterpret_cast<uintptr_t>(p.biases) & 15)))
    pl.sct = false;
  if (!pl.sct && pl.engine != 0) pl = plan_mma(p.N, p.K, p.bits, epi, epi == EPI_QKROPE ? 128 : 0, rt);
  if (p.x_seg != 0 || p.ssq_seg != 0) {
    if (pl.engine != 2)
      return fail(DSPARK_ERR_UNSUPPORTED, "qmm: segmented x rows need the streaming engine (K %% 512 == 0)");
    if (p.x_seg % 8 || p.x_segstride % 8 || p.x_seg <= 0)
      return fail(DSPARK_ERR_UNSUPPORTED, "qmm: x segments must be multiples of 8 elements");
  }
  if ((p.peer_world > 0 || p.wait_flag != nullptr) && (pl.engine != 2 || pl.tcmma))
    return fail(DSPARK_ERR_UNSUPPORTED,
                "qmm: peer stores / gather waits need the streaming engine with mma.sync consumers");
  if (pl.halves && p.M > 16 && p.peer_world == 0 && p.wait_flag == nullptr) {
    // two launches of the 16-row plan: every per-row pointer of the second one moves 16 rows
    // (x, out, residual, statistics in / out, q output, positions, cache offsets)
    const QmmPlan h = plan(p.N, p.K, p.bits, epi, epi == EPI_QKROPE ? 128 : 0, 2);
    if (h.nw != 0 && !h.halves) {
      QmmParams a = p_in;
      a.M = 16;
      const int rc = run(a, epi, &h, stream);
      if (rc != DSPARK_OK) return rc;
      QmmParams b = p_in;
      b.M = p_in.M - 16;
      b.x = p_in.x + 16 * p_in.ldx;
      if (b.out) b.out = p_in.out + 16 * p_in.ldo;
      if (b.resid) b.resid = p_in.resid + 16 * p_in.ldr;
      if (b.ssq_in) b.ssq_in = p_in.ssq_in + 16;
      if (b.ssq_out) b.ssq_out = p_in.ssq_out + 16;
      if (b.qout) b.qout = p_in.qout + 16 * p_in.ldq;
      if (b.row_pos) b.row_pos = p_in.row_pos + 16;
      if (b.row_kv) b.row_kv = p_in.row_kv + 16;
      return run(b, epi, &h, stream);
    }
  }
  p.kslice = pl.kslice;
  p.cs = pl.cs;
  p.nslots = pl.nslots;
  if (pl.engine == 2) return run_st(p, epi, pl, stream);
  if (pl.engine == 1) return run_tc(p, epi, pl, stream);
  if (p.bits == 4) {
    switch (epi) {
      case EPI_PLAIN: return dispatch_rt<4, EPI_PLAIN>(p, pl, stream);
      case EPI_RESID: return dispatch_rt<4, EPI_RESID>(p, pl, stream);
      case EPI_SWIGLU: return dispatch_rt<4, EPI_SWIGLU>(p, pl, stream);
      case EPI_QKROPE: return dispatch_rt<4, EPI_QKROPE>(p, pl, stream);
    }
  } else {
    switch (epi) {
      case EPI_PLAIN: return dispatch_rt<8, EPI_PLAIN>(p, pl, stream);
      case EPI_RESID: return dispatch_rt<8, EPI_RESID>(p, pl, stream);
      case EPI_SWIGLU: return dispatch_rt<8, EPI_SWIGLU>(p, pl, stream);
      case EPI_QKROPE: return dispatch_rt<8, EPI_QKROPE>(p, pl, stream);
    }
  }
  return fail(DSPARK_ERR_ARG, "qmm: bad epilogue %d", epi);
}

}  // namespace qmm
}  // namespace dspark
