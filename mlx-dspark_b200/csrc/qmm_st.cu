// K1, streaming engine: small-M affine-quantized matmul y[M,N] = x[M,K] . dequant(W)^T for
// 1-32 rows (sm_100a). Same contract and numerics as qmm.cu / qmm_tc.cu (MLX affine 4/8-bit,
// group 64, fp32 accumulation, per-group scale/bias fold, bf16 out) and the same epilogues.
//
// Why a third engine. At M <= 32 the product is ~64 flop per weight byte: HBM-bound by a
// wide margin, and the tensor core is never the limit. What limits a CTA is how fast it can
// turn packed weights into MMA operands and fold each group's product with its scale. This
// engine keeps that chain — shared-memory load, dequantize, MMA, fold — inside each warp, so
// the only synchronisation on the weight stream is the TMA ring itself:
//
//  * Persistent clusters (grid (cs, P)): the cs CTAs of a cluster split K; P clusters walk the
//    128-row output tiles t = cluster, cluster + P, ... One producer warp streams each CTA's
//    weights through a ring of 16 KB stages (one 128-byte x 128-row TMA box, 128-byte swizzle,
//    L2 evict-first); every 8 groups the scales and biases ride on the same mbarrier. The
//    producer never waits on the previous kernel (griddepcontrol.wait), so under programmatic
//    dependent launch a kernel's first weight stages stream while its predecessor finishes.
//  * Eight consumer warps, each owning 32 tile rows (two 16-row MMA groups sharing one set of x
//    fragments) and one k half of every stage. Per group of 64 k a thread loads its rows' words
//    (one 8- or 16-byte ld.shared each, conflict-free through a row permutation matched to the
//    swizzle), dequantizes them with the bf16 magic-exponent trick (nibble | 0x4300 = 128 + q,
//    exact; 8-bit as two exact nibble planes 128 + lo and 256 + 16 hi) straight into mma.m16n8k16
//    A fragments (the weights are the 16-row A operand, x the 8-column B operand, so every
//    weight is read once whatever M is), and folds the group's exact product P into fp32
//    accumulators: acc += scale*P + (bias - MAGIC*scale) * sum_k x (packed f32x2 FMAs).
//  * x (the CTA's K slice, <= 32 rows) is staged once per launch by the epilogue warps, which
//    are idle until the first tile ends: 512 k at a time (16-byte global loads, 8 in flight per
//    thread), normed, k permuted inside each 8-block (4-bit) or 4-block (8-bit) exactly as the
//    magic extraction orders the weights, and summed per group, each block released on its own
//    mbarrier. The first tile's consumers wait per block, so staging overlaps their compute;
//    one 16-byte load gives the B fragments of two k16 steps.
//  * Four epilogue warps finish each tile while the consumers stream the next one. At a tile's
//    end every consumer warp pushes its k half of the partial tile to the rows' owners (row m
//    belongs to cluster rank m % cs) and goes straight on: st.async into a peer's receive
//    buffer (the peer's mbarrier counts the bytes; no fence, no handshake), plain stores and a
//    per-warp arrive for its own rows. The owner sums the halves of each rank, then the ranks,
//    in fixed order (double-buffered; deterministic, and a row's result never depends on how
//    many rows ride with it), then the shared epilogue runs on them.
//  * tcgen05 consumers (template flag TC, DSPARK_QMM_ST_TC=1): eight dequantization warps write
//    each row's weights fully dequantized (w = scale * q + bias, one rounding to bf16) into
//    double-buffered A buffers in tensor memory, one MMA warp accumulates the whole K slice of
//    a tile into a D buffer (M = 128 tile rows, N = 16 or 32 staged x rows), and the epilogue
//    warps read D once per tile and push it like the partials above. Correct (row-count
//    invariant within a row class) but slower at these row counts, for a measured reason: on
//    B200 one kind::f16 MMA with M = 128, K = 16 takes ~100-150 SM cycles whatever N is up to
//    128 and however many independent accumulators are in flight, i.e. the tensor core takes in
//    only ~20 weights per cycle as the 128-row A operand, where HBM delivers ~45 per cycle per
//    SM; mma.m16n8k16 with the weights as the 16-row A operand takes in ~59 per cycle at 16 rows
//    (microbenchmarks, 2026-12-02). The same consumers are the right shape once x has 128+ rows.
// Every mbarrier wait is time-bounded (a failed wait records an error in the device status word
// and the kernel drains without further waits on other agents).
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "host_common.h"
#include "qmm.h"
#include "qmm_epilogue.cuh"
#include "tcgen05.cuh"

namespace dspark {
namespace qmm {
namespace st {

constexpr int TN = 128;                 // weight rows per tile
constexpr int NWC = 8;                  // consumer warps, 16 weight rows each
constexpr int WARP_TMA = NWC;           // the producer warp
constexpr int NWE = 4;                  // epilogue warps
constexpr int WARP_EPI = NWC + 1;
constexpr int NTHR = (NWC + 1 + NWE) * 32;
constexpr int WARP_MMA = NWC + 1 + NWE;  // tcgen05 engine: the MMA-issuing warp
constexpr int NTHR_TC = NTHR + 32;
constexpr int NC = NWC * 32;
constexpr int NE = NWE * 32;
constexpr int PSTR = TN + 4;            // fp32 row stride of partial / reduced tiles
constexpr int STG = TN * 128;           // one stage: a 128-byte-wide box of 128 rows
constexpr int SCB = TN * 16;            // 8 groups of bf16 scales (or biases) for 128 rows
constexpr int KBLK = 512;               // k per scale block (8 groups)
constexpr int kTcBars = 16;             // tcgen05 engine barriers (A full / empty, D full / empty)
constexpr int kXBlocks = 16;            // x staging blocks of 512 k per K slice (kslice <= 8192)

template <int BITS>
struct Tr;
template <>
struct Tr<4> {
  static constexpr int KB = 256;   // k per stage
  static constexpr int GPS = 4;    // groups per stage
  static constexpr int SPS = 2;    // stages per scale block
  static constexpr float MAGIC = 128.0f;
};
template <>
struct Tr<8> {
  static constexpr int KB = 128;
  static constexpr int GPS = 2;
  static constexpr int SPS = 4;
  static constexpr float MAGIC = 384.0f;  // 128 (low plane) + 256 (high plane)
};

// Scale-block slots: block b (stages b*SPS .. b*SPS+SPS-1) is reloaded into its slot only
// after stage b*SPS + SPS - 1 has been consumed, which the weight ring guarantees when
// SS * SPS >= S + SPS - 1.
__host__ __device__ inline int scale_slots(int bits, int nslots) {
  const int sps = bits == 4 ? 2 : 4;
  return (nslots + 2 * sps - 2) / sps;
}

struct Layout {
  int ring, sring, xs, nw, sx, part, red, rs, bars, total;
};

__host__ __device__ inline int x_pitch(int kslice) { return kslice * 2 + 16; }

// Rows of the split-K receive buffer: CTA c of the cluster owns rows m = c + i*cs; every CTA
// pushes its partial rows (one per k half of the tile) into slot [rank][half][i] of the owner.
__host__ __device__ inline int owned_rows(int rp, int cs) { return (rp + cs - 1) / cs; }

// x rows the tcgen05 MMA reads as its N dimension (zero padded): 16 or 32
__host__ __device__ inline int tc_rows(int mt) { return mt <= 2 ? 16 : 32; }

__host__ __device__ inline Layout layout(int bits, int mt, int kslice, int nslots, int cs, bool tc) {
  const int rp = 8 * mt;
  Layout L;
  int off = 0;
  L.ring = off;                      // 1024-byte aligned stages (128-byte swizzle atoms)
  off += nslots * STG;
  L.sring = off;
  off += scale_slots(bits, nslots) * 2 * SCB;
  L.xs = off;  // row-major rows of XP bytes (mma.sync), or 8-k blocks of tc_rows rows (tcgen05)
  off += tc ? (kslice / 8) * tc_rows(mt) * 16 : rp * x_pitch(kslice);
  off = (off + 15) & ~15;
  L.nw = off;  // (unused)
  L.sx = off;
  off += (kslice / 64) * rp * 4;
  off = (off + 15) & ~15;
  L.part = off;  // two receive buffers [cs sources][2 k halves][owned_rows][PSTR]
  off += 2 * cs * 2 * owned_rows(rp, cs) * PSTR * 4;
  L.red = off;
  off += rp * PSTR * 4;
  L.rs = off;
  off += 32 * 4;
  off = (off + 15) & ~15;
  L.bars = off;
  off += (2 * nslots + 4 + kXBlocks + kTcBars) * 8 + 16;  // + x blocks, tcgen05, TMEM slot
  L.total = off + 1024;  // slack to align the dynamic base to 1024 bytes
  return L;
}

// Physical tile row of MMA row g (0..7) inside a 16-row group. The 128-byte swizzle stores
// 16-byte chunk c of row r at chunk c ^ (r & 7); these permutations make the rows that one
// shared-memory wavefront serves (4 rows for 8-byte loads, 2 rows for 16-byte loads) land on
// disjoint chunks, so the weight loads are bank-conflict free.
template <int BITS>
__device__ __forceinline__ int row_perm(int g) {
  return BITS == 4 ? (((g & 3) << 1) | (g >> 2)) : (((g & 1) << 2) | (g >> 1));
}

// bf16x2 helpers of the tcgen05 dequantization (round to nearest once per result)
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
// the bf16 of group g of a block's 8 packed values, in both halves
__device__ __forceinline__ uint32_t bf2_dup(uint4 v, int g) {
  const int w = g >> 1;
  const uint32_t x = w == 0 ? v.x : w == 1 ? v.y : w == 2 ? v.z : v.w;
  return __byte_perm(x, 0u, (g & 1) ? 0x3232u : 0x1010u);
}

// tcgen05 engine, dequantization warps (two warpgroups of 4). Thread t of warp w owns tile row
// r = 32 * (w % 4) + t == TMEM lane r; warpgroup wg takes the k half wg of every stage (64 bytes
// of the row). Per stage it loads those bytes from the ring (four conflict-free 16-byte loads
// through the 128-byte swizzle), releases the slot, and writes the row's weights fully
// dequantized, w = scale * q + bias rounded once to bf16 (q = (128 + q) - 128 exactly from the
// magic-exponent extraction, then one bf16x2 FMA), into one of its two A buffers in tensor
// memory, in the k order the staged x uses (4-bit: 0,4,1,5,2,6,3,7 inside each 8-block; 8-bit:
// 0,2,1,3 inside each 4-block, q = lo + 16 hi exactly). The MMA warp's commit frees a buffer.
template <int BITS>
__device__ __forceinline__ void dequant_tc(const QmmParams& p, uint8_t* ring, uint8_t* sring,
                                           uint64_t* full, uint64_t* empty, uint64_t* afull,
                                           uint64_t* aempty, uint32_t tmem, int ntl, int nsb,
                                           int S, int SS, bool& ok) {
  constexpr int SPS = Tr<BITS>::SPS;
  constexpr int GPS = Tr<BITS>::GPS;
  constexpr int ACOLS = BITS == 4 ? 64 : 32;  // TMEM columns of a half stage (2 bf16 each)
  constexpr uint32_t M128 = 0x43004300u;      // (128, 128) in bf16x2
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wg = warp >> 2, wq = warp & 3;
  const int row = wq * 32 + lane;
  const uint32_t ta = tmem + (uint32_t(wq * 32) << 16) + uint32_t(wg * 2 * ACOLS);
  const uint32_t ring_a = smem_u32(ring);
  const uint32_t sring_a = smem_u32(sring);
  int g = 0, slot = 0, phase = 0, sslot = 0;
  for (int j = 0; j < ntl; ++j) {
    for (int sb = 0; sb < nsb; ++sb) {
      uint4 sv4 = make_uint4(0u, 0u, 0u, 0u), bv4 = sv4;
#pragma unroll 1
      for (int si = 0; si < SPS; ++si, ++g) {
        if (ok) ok = mbar_wait(&full[slot], uint32_t(phase), p.status, kErrWaitFull);
        if (si == 0) {  // this row's scales / biases of the block's 8 groups
          const uint32_t sa = sring_a + uint32_t(sslot * 2 * SCB + row * 16);
          sv4 = lds128(sa);
          bv4 = lds128(sa + SCB);
          if (++sslot == SS) sslot = 0;
        }
        uint32_t wd[16];
        const uint32_t wrow = ring_a + uint32_t(slot * STG + row * 128);
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const uint4 v = lds128(wrow + uint32_t(((4 * wg + h) ^ (row & 7)) << 4));
          wd[4 * h + 0] = v.x; wd[4 * h + 1] = v.y; wd[4 * h + 2] = v.z; wd[4 * h + 3] = v.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);  // the stage's bytes are in registers
        if (++slot == S) {
          slot = 0;
          phase ^= 1;
        }
        const int ab = g & 1;
        // the MMAs that read buffer ab two stages ago are done
        if (g >= 2 && ok)
          ok = mbar_wait(&aempty[wg * 2 + ab], uint32_t(((g - 2) >> 1) & 1), p.status, kErrWaitMma);
        tcg::tc_fence_after();
        const uint32_t dst = ta + uint32_t(ab * ACOLS);
        uint32_t r[32];
        if (BITS == 4) {
          // two groups of 8 words; word u, nibbles e and e + 4 -> column 4u + e
#pragma unroll
          for (int gg = 0; gg < 2; ++gg) {
            const int gb = si * GPS + wg * 2 + gg;  // group inside the scale block
            const uint32_t s2 = bf2_dup(sv4, gb), b2 = bf2_dup(bv4, gb);
#pragma unroll
            for (int u = 0; u < 8; ++u)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const uint32_t m = lop3_and_or(wd[8 * gg + u] >> (4 * e), 0x000F000Fu, M128);
                r[4 * u + e] = bf2_fma(bf2_sub(m, M128), s2, b2);
              }
            tcg::tmem_st32(dst + uint32_t(32 * gg), r);
          }
        } else {
          // one group of 16 words; word u -> columns 2u (k 0, 2) and 2u + 1 (k 1, 3)
          const int gb = si * GPS + wg;
          const uint32_t s2 = bf2_dup(sv4, gb), b2 = bf2_dup(bv4, gb);
          constexpr uint32_t SIXTEEN = 0x41804180u;  // (16, 16)
#pragma unroll
          for (int u = 0; u < 16; ++u)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const uint32_t x = wd[u] >> (8 * e);
              const uint32_t lo = bf2_sub(lop3_and_or(x, 0x000F000Fu, M128), M128);
              const uint32_t hi = bf2_sub(lop3_and_or(x >> 4, 0x000F000Fu, M128), M128);
              r[2 * u + e] = bf2_fma(bf2_fma(hi, SIXTEEN, lo), s2, b2);
            }
          tcg::tmem_st32(dst, r);
        }
        tcg::tmem_wait_st();
        tcg::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[wg * 2 + ab]);
      }
    }
  }
}

// tcgen05 engine, MMA warp (one elected thread): per stage, once both warpgroups' A buffers are
// written, the stage's MMAs (M = 128 tile rows from tensor memory, N = NM staged x rows from
// shared memory, K = 16 each) accumulate into the tile's D buffer; a commit per buffer frees it
// for the dequantization warps, and a commit at the tile's end hands D to the epilogue warps.
// D is double-buffered, so tile j + 1 accumulates while tile j is read out. The first tile also
// waits until the epilogue warps have staged each 512-k block of x.
template <int BITS, int NM>
__device__ __forceinline__ void mma_tc(const QmmParams& p, uint8_t* xs, uint64_t* afull,
                                       uint64_t* aempty, uint64_t* dfull, uint64_t* dempty,
                                       uint64_t* xrdy, uint64_t* mfin, uint32_t tmem, int ntl,
                                       int nst, bool& ok) {
  constexpr int KB = Tr<BITS>::KB;
  constexpr int ACOLS = BITS == 4 ? 64 : 32;
  constexpr int MPH = ACOLS / 8;  // MMAs per half stage
  constexpr uint32_t IDESC = tcg::idesc_bf16(NM);
  constexpr uint32_t DCOL = 4 * ACOLS;  // D buffers after the four A buffers
  if (tcg::elect_one()) {
    const uint64_t bd0 = tcg::smem_desc(smem_u32(xs), NM * 16, 128);
    int g = 0;
    bool issued = false;
    for (int j = 0; j < ntl && ok; ++j) {
      const int db = j & 1;
      if (j >= 2) ok = mbar_wait(&dempty[db], uint32_t(((j - 2) >> 1) & 1), p.status, kErrWaitMma);
      tcg::tc_fence_after();
      const uint32_t dd = tmem + DCOL + uint32_t(db * NM);
      for (int st = 0; st < nst && ok; ++st, ++g) {
        if (j == 0 && (st * KB) % KBLK == 0)
          ok = mbar_wait(&xrdy[(st * KB) / KBLK], 0, p.status, kErrWaitFull);
        const int ab = g & 1;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (ok) ok = mbar_wait(&afull[h * 2 + ab], uint32_t((g >> 1) & 1), p.status, kErrWaitMma);
          if (!ok) break;
          tcg::tc_fence_after();
          const uint32_t aa = tmem + uint32_t((h * 2 + ab) * ACOLS);
#pragma unroll
          for (int s = 0; s < MPH; ++s) {
            const int kk = st * KB + h * (KB / 2) + 16 * s;
            tcg::umma_ts(dd, aa + uint32_t(8 * s), bd0 + uint64_t((kk / 8) * NM), IDESC,
                         (st | h | s) ? 1u : 0u);
          }
          tcg::umma_commit(&aempty[h * 2 + ab]);
          issued = true;
        }
      }
      if (ok) tcg::umma_commit(&dfull[db]);
    }
    // no MMA may still write tensor memory when the CTA releases it
    if (issued) {
      tcg::umma_commit(mfin);
      mbar_wait(mfin, 0, p.status, kErrWaitMma);
    }
  }
  __syncwarp();
}

// Stage k block kb of x for the tcgen05 engine: like stage_block, but every chunk lands in the
// K-major canonical layout the MMA reads (8-k block c of row m at (c * NM + m) * 16), rows
// M .. NM - 1 are zero-filled, and no group sums are kept (the weights arrive dequantized).
template <int BITS, int NM, int U>
__device__ __forceinline__ void stage_block_tc(const QmmParams& p, uint8_t* xs, const float* rsm,
                                               bool nrm, int kbase, int kb, int t) {
  const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
  const int c = kb * 64 + (t & 63);
  const int k = kbase + c * 8;
  const int xseg = int(p.x_seg);
  int seg = 0, off = k;
  if (xseg) {
    seg = off / xseg;
    off -= seg * xseg;
  }
  const bf16* col = p.x + long(seg) * p.x_segstride + off;
  const uint4 w = nrm ? ldg_v4(p.norm_w + k) : z4;
  const uint32_t* pw = reinterpret_cast<const uint32_t*>(&w);
  for (int m0 = t >> 6; m0 < NM; m0 += 2 * U) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      v[u] = m0 + 2 * u < p.M ? ldcg_v4(col + (size_t)(m0 + 2 * u) * p.ldx) : z4;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int m = m0 + 2 * u;
      if (m >= NM) break;
      uint4 vv = v[u];
      uint32_t* pv = reinterpret_cast<uint32_t*>(&vv);
      if (nrm && m < p.M) {
        const float r = rsm[m];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          pv[e] = pack_bf16x2(bf16_lo(pv[e]) * r * bf16_lo(pw[e]),
                              bf16_hi(pv[e]) * r * bf16_hi(pw[e]));
      }
      uint4 o;
      if (BITS == 4) {
        o.x = __byte_perm(vv.x, vv.z, 0x5410);
        o.y = __byte_perm(vv.x, vv.z, 0x7632);
        o.z = __byte_perm(vv.y, vv.w, 0x5410);
        o.w = __byte_perm(vv.y, vv.w, 0x7632);
      } else {
        o.x = __byte_perm(vv.x, vv.y, 0x5410);
        o.y = __byte_perm(vv.x, vv.y, 0x7632);
        o.z = __byte_perm(vv.z, vv.w, 0x5410);
        o.w = __byte_perm(vv.z, vv.w, 0x7632);
      }
      *reinterpret_cast<uint4*>(xs + (size_t(c) * NM + m) * 16) = o;
    }
  }
}

// rs[m] = rsqrt(mean of x_m^2 + eps) for rows m = m0, m0 + mstep, ... from the sums of squares
// the previous projection's epilogue left per tile (segmented when gathered from several ranks).
// Entry e = lane + 32i lives in segment e / ssq_seg: advanced by subtraction, so no division
// sits between the loads. One warp per row.
__device__ __forceinline__ void norm_stats(const QmmParams& p, float* rsm, int rp, int m0,
                                           int mstep, int lane) {
  // every row's loads are issued before any reduction (one global-memory latency in all, not
  // one per row); each row's entries are still summed in the same order (lane-strided, then a
  // fixed shuffle tree), so the result is unchanged
  constexpr int MAXR = 8;  // rows per warp: rp <= 32 rows over mstep >= 4 warps
  float ss[MAXR];
#pragma unroll
  for (int i = 0; i < MAXR; ++i) ss[i] = 0.f;
  const int sg = p.ssq_seg;
  int sseg = 0, soff = lane;
  if (sg) {
    sseg = lane / sg;
    soff = lane - sseg * sg;
  }
  for (int e = lane; e < p.ssq_n; e += 32) {
    const long at = sg ? sseg * p.ssq_segstride + long(soff) * p.ssq_stride
                       : long(e) * p.ssq_stride;
#pragma unroll
    for (int i = 0; i < MAXR; ++i) {
      const int m = m0 + i * mstep;
      if (m < rp && m < p.M) ss[i] += __ldcg(&p.ssq_in[at + m]);
    }
    soff += 32;
    if (sg)
      while (soff >= sg) {
        soff -= sg;
        ++sseg;
      }
  }
#pragma unroll
  for (int i = 0; i < MAXR; ++i) {
    const int m = m0 + i * mstep;
    float v = ss[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0 && m < rp) rsm[m] = m < p.M ? rsqrtf(v / float(p.K) + p.eps) : 0.f;
  }
}

// Row width (floats, a multiple of 4) of the statistics block staged by norm_stats_staged, or 0
// when the block does not qualify (segmented, unaligned, or larger than the scratch).
__device__ __forceinline__ int ssq_stage_width(const QmmParams& p, int rp, int scratch_floats) {
  const int w = (min(p.M, rp) + 3) & ~3;
  if (p.ssq_seg || (reinterpret_cast<uintptr_t>(p.ssq_in) & 15) || (p.ssq_stride & 3) ||
      w > p.ssq_stride || p.ssq_n * w > scratch_floats)
    return 0;
  return w;
}

// norm_stats for a contiguous statistics block. The block (ssq_n entries x the launch's rows, a
// few KB) is read by every CTA of the launch at the same moment; per-row strided loads made
// hundreds of line requests per CTA, which queued at the lines' L2 slices (measured: ~2.5 us for
// the one round trip). Here the epilogue threads first copy it into shared memory with 16-byte
// loads (a few line requests per CTA), then sums each row from there in the same order as
// norm_stats (lane-strided over entries, then the fixed shuffle tree): the same rs bits.
__device__ __forceinline__ void norm_stats_staged(const QmmParams& p, float* rsm, int rp, int w,
                                                  float* scratch, int etid) {
  const int w4 = w / 4;
  for (int i = etid; i < p.ssq_n * w4; i += NE) {
    const int e = i / w4, c = i - e * w4;
    *reinterpret_cast<float4*>(&scratch[e * w + c * 4]) =
        __ldcg(reinterpret_cast<const float4*>(&p.ssq_in[long(e) * p.ssq_stride + c * 4]));
  }
  asm volatile("bar.sync 2, %0;" ::"n"(NE));  // the block is staged
  // One thread per row, every row at once (four rows per warp through dependent shuffle chains
  // were measurably slower on this launch-head path). Each of the 32 partials a[l] sums entries
  // l, l + 32, ... in order (a lane's share in norm_stats), and the partials are paired as the
  // xor-shuffle tree pairs lanes (l with l + 16, then l + 8, ...): norm_stats' bits.
  if (etid < rp) {
    const int m = etid;
    float r = 0.f;
    if (m < p.M) {
      float a[32];
#pragma unroll
      for (int l = 0; l < 32; ++l) a[l] = 0.f;
      for (int e0 = 0; e0 < p.ssq_n; e0 += 32) {
#pragma unroll
        for (int l = 0; l < 32; ++l)
          if (e0 + l < p.ssq_n) a[l] += scratch[(e0 + l) * w + m];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int l = 0; l < o; ++l) a[l] += a[l + o];
      }
      r = rsqrtf(a[0] / float(p.K) + p.eps);
    }
    rsm[m] = r;
  }
}

// Stage k block kb (512 k: chunks c = 64kb .. 64kb + 63 of the K slice) of every row of x into
// shared memory (rows of XP bytes). Epilogue warp `we` (of 4) stages the chunks of groups 2we and
// 2we + 1 (16 chunk columns) of every row, which are the groups whose sums it forms next, so a
// warp-level sync is the only one between the two: lane l takes chunk column 64kb + 16we + l % 16
// and rows l / 16, l / 16 + 2, ..., U loads in flight at once (16-byte global loads). Each chunk
// is normed (x * rs * w rounded to bf16) and permuted inside each 8-block (4-bit:
// 0,4,1,5,2,6,3,7) or 4-block (8-bit: 0,2,1,3) as the magic extraction orders the weights. The
// block's one division (the segment of k) comes before its loads are issued.
template <int BITS, int RP, int U>
__device__ __forceinline__ void stage_block(const QmmParams& p, uint8_t* xs, int XP,
                                            const float* rsm, bool nrm, int kbase, int kb, int we,
                                            int lane) {
  const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
  const int c = kb * 64 + 16 * we + (lane & 15);
  const int k = kbase + c * 8;
  const int xseg = int(p.x_seg);
  int seg = 0, off = k;
  if (xseg) {
    seg = off / xseg;
    off -= seg * xseg;
  }
  const bf16* col = p.x + long(seg) * p.x_segstride + off;
  const uint4 w = nrm ? ldg_v4(p.norm_w + k) : z4;
  const uint32_t* pw = reinterpret_cast<const uint32_t*>(&w);
  // row pointers and shared-memory addresses advance by increments (no per-row 64-bit products)
  const size_t rstep = size_t(2) * size_t(p.ldx);
  float wl[4], wh[4];  // the chunk's norm weights, unpacked once
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    wl[e] = bf16_lo(pw[e]);
    wh[e] = bf16_hi(pw[e]);
  }
  for (int m0 = lane >> 4; m0 < p.M; m0 += 2 * U) {  // the row parity of a half-warp
    uint4 v[U];
    const bf16* rp = col + size_t(m0) * size_t(p.ldx);
    const int nu = min(U, (p.M - m0 + 1) >> 1);  // rows of this pass (per half-warp)
#pragma unroll
    for (int u = 0; u < U; ++u) {
      v[u] = u < nu ? ldcg_v4(rp) : z4;
      rp += rstep;
    }
    uint8_t* xp = xs + m0 * XP + c * 16;
#pragma unroll
    for (int u = 0; u < U; ++u, xp += 2 * XP) {
      const int m = m0 + 2 * u;
      if (u >= nu) break;  // uniform in a half-warp
      uint4 vv = v[u];
      uint32_t* pv = reinterpret_cast<uint32_t*>(&vv);
      if (nrm) {  // bf16((x * r) * w), the products in packed pairs
        const float r = rsm[m];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float a0 = bf16_lo(pv[e]), a1 = bf16_hi(pv[e]);
          mul2(a0, a1, r, r);
          mul2(a0, a1, wl[e], wh[e]);
          pv[e] = pack_bf16x2(a0, a1);
        }
      }
      uint4 o;
      if (BITS == 4) {
        o.x = __byte_perm(vv.x, vv.z, 0x5410);
        o.y = __byte_perm(vv.x, vv.z, 0x7632);
        o.z = __byte_perm(vv.y, vv.w, 0x5410);
        o.w = __byte_perm(vv.y, vv.w, 0x7632);
      } else {
        o.x = __byte_perm(vv.x, vv.y, 0x5410);
        o.y = __byte_perm(vv.x, vv.y, 0x7632);
        o.z = __byte_perm(vv.z, vv.w, 0x5410);
        o.w = __byte_perm(vv.z, vv.w, 0x7632);
      }
      *reinterpret_cast<uint4*>(xp) = o;
    }
  }
}

// The per-group sums of a staged k block (8 groups of 64 k, every row), sx[g * RP + m] = sum_k
// x[m, k], on the tensor core: mma.m16n8k16 with an all-ones A operand and the consumers' own x
// fragments as B (two k16 steps per 16-byte load, 8 rows per n tile) sums 16 k of 8 rows per
// instruction, where per-element unpacking and shuffle trees cost ~20 instructions per 16-byte
// chunk of every row in the staging warps. Epilogue warp w (of 4) takes groups 2w, 2w + 1 of the
// block; lanes 0-3 write the rows' sums. Reads the chunks this warp staged (stage_block), after a
// warp-level sync.
template <int RP>
__device__ __forceinline__ void group_sums_mma(const uint8_t* xs, int XP, float* sx, int kb,
                                               int we, int lane) {
  constexpr int MT = RP / 8;
  constexpr uint32_t ONES = 0x3F803F80u;  // bf16 1.0 in both halves
  const int g8 = lane >> 2, t4 = lane & 3;
  const uint32_t xa = smem_u32(xs) + uint32_t(g8 * XP + t4 * 32);
#pragma unroll
  for (int gi = 0; gi < 2; ++gi) {
    const int gl = kb * 8 + we * 2 + gi;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const uint32_t a = xa + uint32_t(mt * 8 * XP + gl * 128);
      const uint4 q0 = lds128(a);
      const uint4 q1 = lds128(a + 16);
      // two independent accumulation chains (k 0-31 and 32-63 of the group), then their sum
      float d[4] = {0.f, 0.f, 0.f, 0.f}, e[4] = {0.f, 0.f, 0.f, 0.f};
      mma_bf16_16816(d, ONES, ONES, ONES, ONES, q0.x, q0.y);
      mma_bf16_16816(e, ONES, ONES, ONES, ONES, q1.x, q1.y);
      mma_bf16_16816(d, ONES, ONES, ONES, ONES, q0.z, q0.w);
      mma_bf16_16816(e, ONES, ONES, ONES, ONES, q1.z, q1.w);
      if (g8 == 0)
        *reinterpret_cast<float2*>(sx + gl * RP + mt * 8 + 2 * t4) =
            make_float2(d[0] + e[0], d[1] + e[1]);
    }
  }
}

template <int BITS, int MT, int EPI, bool TC, bool PEER = false>
__global__ void __launch_bounds__(TC ? NTHR_TC : NTHR, 1)
    qmm_st_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
                  const __grid_constant__ CUtensorMap bmap, const QmmParams p) {
  constexpr int RP = 8 * MT;
  constexpr int KB = Tr<BITS>::KB;
  constexpr int GPS = Tr<BITS>::GPS;
  constexpr int SPS = Tr<BITS>::SPS;
  constexpr float MAGIC = Tr<BITS>::MAGIC;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align_up<1024>(smem_raw);
  const int S = p.nslots;
  const int SS = scale_slots(BITS, S);
  const Layout Lo = layout(BITS, MT, p.kslice, S, p.cs, TC);
  uint8_t* ring = smem + Lo.ring;
  uint8_t* sring = smem + Lo.sring;
  uint8_t* xs = smem + Lo.xs;
  float* sx = reinterpret_cast<float*>(smem + Lo.sx);
  float* part = reinterpret_cast<float*>(smem + Lo.part);
  float* red = reinterpret_cast<float*>(smem + Lo.red);
  float* rsm = reinterpret_cast<float*>(smem + Lo.rs);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lo.bars);
  uint64_t* empty = full + S;
  uint64_t* ready = empty + S;   // [2] every local warp and every peer's bytes of a partial tile
  uint64_t* freeb = ready + 2;   // [2] every cluster CTA finished reading this CTA's partial
  uint64_t* xrdy = freeb + 2;    // [kXBlocks] k block b of the x slice is staged
  uint64_t* tcbar = xrdy + kXBlocks;  // tcgen05 engine:
  uint64_t* afull = tcbar;            // [2 warpgroups][2] A buffer written (4 warp arrivals)
  uint64_t* aempty = tcbar + 4;       // [2][2] the MMAs reading it are done (commit)
  uint64_t* dfull = tcbar + 8;        // [2] the tile's D is complete (commit)
  uint64_t* dempty = tcbar + 10;      // [2] the epilogue warps have read D (NWE arrivals)
  uint64_t* mfin = tcbar + 12;        // the MMA warp's last commit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tcbar + kTcBars);

  const int cs = p.cs;
  const int rank = blockIdx.x;
  const int ntiles = (p.N + TN - 1) / TN;
  const int nclus = gridDim.y;
  const int ntl = int(blockIdx.y) < ntiles ? (ntiles - int(blockIdx.y) + nclus - 1) / nclus : 0;
  const int kbase = rank * p.kslice;
  const int kvalid = min(p.kslice, p.K - kbase);
  const int nsb = (kvalid + KBLK - 1) / KBLK;  // scale blocks per tile (K % 512 == 0)
  const int nst = nsb * SPS;                    // stages per tile
  const int XP = x_pitch(p.kslice);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tid = threadIdx.x;

  if (warp == WARP_TMA && lane == 0) {  // descriptor fetches overlap the set-up
    prefetch_tmap(&wmap);
    prefetch_tmap(&smap);
    prefetch_tmap(&bmap);
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NWC);
    }
    for (int i = 0; i < 2; ++i) {
      // the owner's expect-tx arrive (peers' st.async bytes) + one arrive per local warp that
      // stores partial rows (the consumers, or with tcgen05 the epilogue warps reading D)
      mbar_init(&ready[i], 1 + (TC ? NWE : NWC));
      mbar_init(&freeb[i], cs);
    }
    // x block staged: one arrive per epilogue warp after its group sums (mma.sync engine), or
    // one after the block's barrier (tcgen05 engine)
    for (int i = 0; i < kXBlocks; ++i) mbar_init(&xrdy[i], TC ? 1 : NWE);
    for (int i = 0; i < kTcBars; ++i) mbar_init(&tcbar[i], 1);
    if (TC) {
      for (int i = 0; i < 4; ++i) mbar_init(&afull[i], 4);
      for (int i = 0; i < 2; ++i) mbar_init(&dempty[i], NWE);
    }
    fence_mbar_init();
  }
  if constexpr (TC) {
    if (warp == 0) tcg::tmem_alloc(tmem_slot, 512);
    tcg::tc_fence_before();
  }
  __syncthreads();  // this CTA's barriers exist; the producer may start at once
  if constexpr (TC) tcg::tc_fence_after();
  // peers touch this CTA's barriers only after the cluster barrier completes: every thread
  // arrives now and waits right before its first remote access
  if (cs > 1) cluster_arrive();
  pdl_launch_dependents();

  bool ok = true;  // false once a wait on another agent ran out: drain without waiting
  if (warp == WARP_TMA) {
    // ------------------------------------------------------------- producer warp
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int issued = 0;
      int slot = 0, phase = 0, ss = 0;  // ring slot / fill count parity, scale slot
      for (int j = 0; j < ntl && ok; ++j) {
        const int n0 = (int(blockIdx.y) + j * nclus) * TN;
        for (int st = 0; st < nst; ++st) {
          // slot reuse: wait until the consumers released its previous fill
          if (issued >= S && !mbar_wait(&empty[slot], uint32_t(phase ^ 1), p.status, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          const bool sblk = (st % SPS) == 0;
          mbar_arrive_expect_tx(&full[slot], STG + (sblk ? 2 * SCB : 0));
          const int kk = kbase + st * KB;
          tma_load_2d(ring + slot * STG, &wmap, &full[slot], kk * BITS / 32, n0, pol);
          if (sblk) {
            tma_load_2d(sring + ss * 2 * SCB, &smap, &full[slot], kk / 64, n0, pol);
            tma_load_2d(sring + ss * 2 * SCB + SCB, &bmap, &full[slot], kk / 64, n0, pol);
            if (++ss == SS) ss = 0;
          }
          ++issued;
          if (++slot == S) {
            slot = 0;
            phase ^= 1;
          }
        }
      }
      // never leave the CTA with copies in flight: wait (bounded) for the last ones issued
      for (int g = max(0, issued - S); g < issued; ++g)
        mbar_wait(&full[g % S], (g / S) & 1, p.status, kErrWaitFull);
    }
    __syncwarp();
    if (cs > 1) cluster_wait();
    if (!TC && cs > 1) cluster_arrive();  // the exit barrier: no remote access from here on
  } else if (TC && warp < NWC) {
    // ------------------------------------------------------------- tcgen05: dequantization
    dequant_tc<BITS>(p, ring, sring, full, empty, afull, aempty, *tmem_slot, ntl, nsb, S, SS, ok);
    if (cs > 1) cluster_wait();
  } else if (TC && warp == WARP_MMA) {
    // ------------------------------------------------------------- tcgen05: MMA issue
    mma_tc<BITS, (MT <= 2 ? 16 : 32)>(p, xs, afull, aempty, dfull, dempty, xrdy, mfin, *tmem_slot,
                                      ntl, nst, ok);
    if (cs > 1) cluster_wait();
  } else if (warp < NWC) {
    // ------------------------------------------------------------- consumer warps (mma.sync)
    const int chunks = p.kslice / 8;
    for (int idx = tid; idx < (RP - p.M) * chunks; idx += NC) {
      const int m = p.M + idx / chunks, c = idx % chunks;
      *reinterpret_cast<uint4*>(xs + m * XP + c * 16) = make_uint4(0u, 0u, 0u, 0u);
    }
    for (int idx = tid; idx < (RP - p.M) * (kvalid / 64); idx += NC) {
      const int g = idx / (RP - p.M), m = p.M + idx % (RP - p.M);
      sx[g * RP + m] = 0.f;
    }
    // the epilogue warps stage x block by block (xrdy); the first tile waits for each block
    asm volatile("bar.sync 1, %0;" ::"n"(NC));

    // Warp w owns 32 tile rows (two 16-row MMA groups sharing one set of x fragments) and one
    // k half of every stage (GH of its GPS groups); the two halves are summed at the tile end.
    constexpr int GH = GPS / 2;
    const int half = warp >> 2, wr = warp & 3;
    const int g8 = lane >> 2, t4 = lane & 3;
    int rows[2][2];
#pragma unroll
    for (int rg = 0; rg < 2; ++rg) {
      rows[rg][0] = wr * 32 + rg * 16 + row_perm<BITS>(g8);
      rows[rg][1] = rows[rg][0] + 8;
    }
    const uint32_t ring_a = smem_u32(ring);
    const uint32_t sring_a = smem_u32(sring);
    // this thread's B fragments of group gl, n8 tile mt: 32 bytes at row (8*mt + g8), k = 16*t4
    const uint32_t xa = smem_u32(xs) + uint32_t(g8 * XP + t4 * 32);
    // swizzled byte offset of (row, logical 16-byte chunk c) inside a stage
    auto wofs = [](int row, int c) { return uint32_t(row * 128 + ((c ^ (row & 7)) << 4)); };
    // 4-bit: the thread's weight offsets inside a stage are the same every stage (row group,
    // row half, group of the warp's k half): computed once, not per load
    uint32_t woff[2][2][GH];
#pragma unroll
    for (int rg = 0; rg < 2; ++rg)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int gg = 0; gg < GH; ++gg)
          woff[rg][h][gg] = BITS == 4 ? wofs(rows[rg][h], (half * GH + gg) * 2 + (t4 >> 1)) +
                                            uint32_t((t4 & 1) * 8)
                                      : 0u;

    // ring slot and phase of the next stage, scale slot of the next block (counted, not divided)
    int slot = 0, phase = 0, sslot = 0;
    for (int j = 0; j < ntl; ++j) {
      float acc[2][MT][4];
#pragma unroll
      for (int rg = 0; rg < 2; ++rg)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[rg][mt][i] = 0.f;

      for (int sb = 0; sb < nsb; ++sb) {
        // the first tile waits until the epilogue warps staged this k block of x
        if (j == 0 && ok) ok = mbar_wait(&xrdy[sb], 0, p.status, kErrWaitFull);
        const uint32_t sblk_a = sring_a + uint32_t(sslot * 2 * SCB);
        if (++sslot == SS) sslot = 0;
#pragma unroll
        for (int si = 0; si < SPS; ++si) {
          const int st = sb * SPS + si;
          if (ok) ok = mbar_wait(&full[slot], uint32_t(phase), p.status, kErrWaitFull);
          // scales / biases of this stage's groups for the thread's 4 rows: one 32-bit word
          // (two consecutive groups) per row
          const int gw = (si * GPS + half * GH) & ~1;  // first group of the word
          const uint32_t sa = sblk_a + uint32_t(gw * 2);
          uint32_t sw[2][2], bw[2][2];
#pragma unroll
          for (int rg = 0; rg < 2; ++rg)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              sw[rg][h] = lds32(sa + rows[rg][h] * 16);
              bw[rg][h] = lds32(sa + SCB + rows[rg][h] * 16);
            }
          const uint32_t wb = ring_a + uint32_t(slot * STG);
#pragma unroll
          for (int gg = 0; gg < GH; ++gg) {
            const int gi = half * GH + gg;     // group inside the stage
            const int gl = st * GPS + gi;      // group inside the K slice
            // which half of the scale word holds this group
            const bool hi16 = ((si * GPS + gi) & 1) != 0;
            // B fragments (x), two k16 steps per 16-byte load, shared by both row groups
            uint32_t b[MT][4][2];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              const uint32_t a = xa + uint32_t(mt * 8 * XP + gl * 128);
              const uint4 q0 = lds128(a);
              const uint4 q1 = lds128(a + 16);
              b[mt][0][0] = q0.x; b[mt][0][1] = q0.y;
              b[mt][1][0] = q0.z; b[mt][1][1] = q0.w;
              b[mt][2][0] = q1.x; b[mt][2][1] = q1.y;
              b[mt][3][0] = q1.z; b[mt][3][1] = q1.w;
            }
#pragma unroll
            for (int rg = 0; rg < 2; ++rg) {
              const int r0 = rows[rg][0], r1 = rows[rg][1];
              float pr[MT][4];
#pragma unroll
              for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int i = 0; i < 4; ++i) pr[mt][i] = 0.f;
              if (BITS == 4) {
                // 8 bytes of each row: group bytes 8*t4 .. 8*t4+7 = k 16*t4 .. 16*t4+15
                const uint2 w0 = lds64(wb + woff[rg][0][gg]);
                const uint2 w1 = lds64(wb + woff[rg][1][gg]);
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                  const uint32_t x0 = (s < 2) ? w0.x : w0.y;
                  const uint32_t x1 = (s < 2) ? w1.x : w1.y;
                  const int e = 2 * (s & 1);
                  const uint32_t a0 = lop3_and_or(x0 >> (4 * e), 0x000F000Fu, 0x43004300u);
                  const uint32_t a2 = lop3_and_or(x0 >> (4 * e + 4), 0x000F000Fu, 0x43004300u);
                  const uint32_t a1 = lop3_and_or(x1 >> (4 * e), 0x000F000Fu, 0x43004300u);
                  const uint32_t a3 = lop3_and_or(x1 >> (4 * e + 4), 0x000F000Fu, 0x43004300u);
#pragma unroll
                  for (int mt = 0; mt < MT; ++mt)
                    mma_bf16_16816(pr[mt], a0, a1, a2, a3, b[mt][s][0], b[mt][s][1]);
                }
              } else {
                // 16 bytes of each row: group bytes 16*t4 .. 16*t4+15 = k 16*t4 .. 16*t4+15
                const int c = gi * 4 + t4;
                const uint4 w0 = lds128(wb + wofs(r0, c));
                const uint4 w1 = lds128(wb + wofs(r1, c));
                const uint32_t wa[4] = {w0.x, w0.y, w0.z, w0.w};
                const uint32_t wc[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                  const uint32_t x0 = wa[s], x1 = wc[s];
                  // low nibble plane: (k0, k2) and (k1, k3) of the word's 4 bytes as 128 + lo
                  uint32_t a0 = lop3_and_or(x0, 0x000F000Fu, 0x43004300u);
                  uint32_t a2 = lop3_and_or(x0 >> 8, 0x000F000Fu, 0x43004300u);
                  uint32_t a1 = lop3_and_or(x1, 0x000F000Fu, 0x43004300u);
                  uint32_t a3 = lop3_and_or(x1 >> 8, 0x000F000Fu, 0x43004300u);
#pragma unroll
                  for (int mt = 0; mt < MT; ++mt)
                    mma_bf16_16816(pr[mt], a0, a1, a2, a3, b[mt][s][0], b[mt][s][1]);
                  // high nibble plane as 256 + 16 hi
                  a0 = lop3_and_or(x0 >> 1, 0x00780078u, 0x43804380u);
                  a2 = lop3_and_or(x0 >> 9, 0x00780078u, 0x43804380u);
                  a1 = lop3_and_or(x1 >> 1, 0x00780078u, 0x43804380u);
                  a3 = lop3_and_or(x1 >> 9, 0x00780078u, 0x43804380u);
#pragma unroll
                  for (int mt = 0; mt < MT; ++mt)
                    mma_bf16_16816(pr[mt], a0, a1, a2, a3, b[mt][s][0], b[mt][s][1]);
                }
              }
              // fold: acc += s*P + (b - MAGIC*s) * sum_k x, rows r0 (i = 0,1) and r1 (i = 2,3)
              const float s0 = hi16 ? bf16_hi(sw[rg][0]) : bf16_lo(sw[rg][0]);
              const float s1 = hi16 ? bf16_hi(sw[rg][1]) : bf16_lo(sw[rg][1]);
              const float c0 = (hi16 ? bf16_hi(bw[rg][0]) : bf16_lo(bw[rg][0])) - MAGIC * s0;
              const float c1 = (hi16 ? bf16_hi(bw[rg][1]) : bf16_lo(bw[rg][1])) - MAGIC * s1;
#pragma unroll
              for (int mt = 0; mt < MT; ++mt) {
                const float2 xs2 = *reinterpret_cast<const float2*>(sx + gl * RP + mt * 8 + 2 * t4);
                fma2(acc[rg][mt][0], acc[rg][mt][1], c0, c0, xs2.x, xs2.y);
                fma2(acc[rg][mt][2], acc[rg][mt][3], c1, c1, xs2.x, xs2.y);
                fma2(acc[rg][mt][0], acc[rg][mt][1], s0, s0, pr[mt][0], pr[mt][1]);
                fma2(acc[rg][mt][2], acc[rg][mt][3], s1, s1, pr[mt][2], pr[mt][3]);
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[slot]);
          if (++slot == S) {
            slot = 0;
            phase ^= 1;
          }
        }
      }

      // ---- push partial tile j (this warp's k half) into receive buffer j & 1 of each row's
      // owner (m % cs), slot [rank][half][m / cs]. Two lanes of the same t4 hold adjacent tile
      // rows 2r and 2r + 1 (g8 and g8 ^ 4 for 4-bit, g8 and g8 ^ 2 for 8-bit: the row
      // permutation) for the same two columns m, m + 1: one exchange gives each lane a row pair
      // for one column, stored with one 8-byte store (st.async to a peer, whose mbarrier counts
      // the bytes; a plain store and a per-warp arrive for this CTA's own rows).
      const int pbuf = j & 1;
      const int ro = owned_rows(RP, cs);
      if (j == 0 && cs > 1) cluster_wait();  // peers' buffers and barriers exist
      // the owners' buffer pbuf last held tile j-2: every owner must be done reading it
      if (j >= 2 && ok)
        ok = mbar_wait_cluster(&freeb[pbuf], ((j - 2) >> 1) & 1, p.status, kErrWaitCluster);
      constexpr int PX = BITS == 4 ? 16 : 8;                     // partner lane mask
      const bool even = BITS == 4 ? (g8 < 4) : ((g8 & 2) == 0);  // this lane holds row 2r
      const uint32_t pa = smem_u32(part + ((pbuf * cs + rank) * 2 + half) * ro * PSTR);
      const uint32_t rb = smem_u32(&ready[pbuf]);
#pragma unroll
      for (int rg = 0; rg < 2; ++rg) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const float* a = acc[rg][mt];  // (r0, m0) (r0, m0+1) (r1, m0) (r1, m0+1)
          const float x0 = __shfl_xor_sync(0xffffffffu, even ? a[1] : a[0], PX);
          const float x1 = __shfl_xor_sync(0xffffffffu, even ? a[3] : a[2], PX);
          const int m = mt * 8 + 2 * t4 + (even ? 0 : 1);
          const int owner = m % cs, ml = m / cs;
          const int r0 = rows[rg][0] & ~1, r1 = rows[rg][1] & ~1;  // first row of each pair
          const float v00 = even ? a[0] : x0, v01 = even ? x0 : a[1];
          const float v10 = even ? a[2] : x1, v11 = even ? x1 : a[3];
          const uint32_t a0 = pa + uint32_t((ml * PSTR + r0) * 4);
          const uint32_t a1 = pa + uint32_t((ml * PSTR + r1) * 4);
          if (owner == rank) {
            asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(a0), "f"(v00), "f"(v01) : "memory");
            asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(a1), "f"(v10), "f"(v11) : "memory");
          } else {
            const uint32_t mb = mapa_shared(rb, owner);
            st_async_v2(mapa_shared(a0, owner), v00, v01, mb);
            st_async_v2(mapa_shared(a1, owner), v10, v11, mb);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ready[pbuf]);  // this warp's local rows are in place
    }
    if (ntl == 0 && cs > 1) cluster_wait();
    // the exit barrier: the last partial is pushed, no remote access from here on
    if (!TC && cs > 1) cluster_arrive();
  } else {
    // ------------------------------------------------------------- epilogue warps
    pdl_wait();  // x, the statistics and the epilogues' buffers come from earlier kernels
    const int etid = tid - WARP_EPI * 32;
    {
      // idle until the first tile ends: stage x for the consumers, 512 k at a time, releasing
      // each block as it lands so that the first tile's compute overlaps the rest
      if (PEER && p.wait_flag != nullptr) {  // x gathered by the producers' peer stores
        if (etid < p.wait_world && ok)
          ok = wait_counter_sys(&p.wait_flag[etid], __ldcg(&p.wait_state[0]) + p.wait_elems,
                                p.status, kErrWaitPeer);
        asm volatile("bar.sync 2, %0;" ::"n"(NE));
      }
      const bool nrm = p.norm_w != nullptr;
      if (nrm) {
        // `red` (the reduced-tile scratch) is free until the first tile's epilogue
        const int sw = ssq_stage_width(p, RP, RP * PSTR);
        if (sw)
          norm_stats_staged(p, rsm, RP, sw, red, etid);
        else
          norm_stats(p, rsm, RP, warp - WARP_EPI, NWE, lane);
        asm volatile("bar.sync 2, %0;" ::"n"(NE));  // rs of every row
      }
      for (int kb = 0; kb < kvalid / KBLK; ++kb) {
        if constexpr (TC) {
          stage_block_tc<BITS, (MT <= 2 ? 16 : 32), 4>(p, xs, rsm, nrm, kbase, kb, etid);
          fence_proxy_async_smem();  // the block becomes the tensor core's B operand
        } else {
          stage_block<BITS, RP, MT == 4 ? 4 : 8>(p, xs, XP, rsm, nrm, kbase, kb, warp - WARP_EPI,
                                                lane);
          __syncwarp();  // this warp's chunks (its two groups, every row) are stored
          group_sums_mma<RP>(xs, XP, sx, kb, warp - WARP_EPI, lane);
          // the warp's chunks and sums are stored: each warp releases its part of the block
          // (the block's barrier counts one arrive per epilogue warp)
          __syncwarp();
          if (lane == 0) mbar_arrive(&xrdy[kb]);
          continue;
        }
        asm volatile("bar.sync 2, %0;" ::"n"(NE));  // the block's chunks are stored
        if (etid == 0) mbar_arrive(&xrdy[kb]);
      }
    }
    if (cs > 1) cluster_wait();  // peers' barriers exist before the first remote arrive
    // the exit barrier's arrive comes after this warp's last remote arrive (the release of tile
    // ntl - 3 below): at once when no tile's buffer is released to a peer
    if (!TC && cs > 1 && ntl < 3) cluster_arrive();
    const int ro = owned_rows(RP, cs);
    const int nmine = (p.M > rank) ? (p.M - rank + cs - 1) / cs : 0;
    // bytes each peer pushes into this CTA per tile: its 2 k halves (one D with tcgen05) of the
    // RP / cs rows m = rank + i*cs this CTA owns (all RP rows are pushed, padding included)
    const int nown = RP > rank ? (RP - rank + cs - 1) / cs : 0;
    constexpr int NHALF = TC ? 1 : 2;
    const uint32_t peer_bytes = uint32_t((cs - 1) * nown * NHALF * TN * 4);
    for (int j = 0; j < ntl; ++j) {
      const int pbuf = j & 1;
      const int t = int(blockIdx.y) + j * nclus;
      const float* pb = part + pbuf * cs * 2 * ro * PSTR;
      // the residual of this tile comes from an earlier kernel: load it before the wait
      uint32_t pre[2 * kResidRows];
      if constexpr (EPI == EPI_RESID) resid_prefetch<TN>(p, rank, cs, t * TN, NWE, WARP_EPI, pre);
      QkPre qk = {};
      if constexpr (EPI == EPI_QKROPE) qkrope_prefetch<TN>(p, rank, cs, NWE, WARP_EPI, qk);
      if constexpr (TC) {
        // read the tile's D (this warp's 32 lanes: tile rows 32 * (warp % 4) + lane, one column
        // per x row), free it for tile j + 2, and push its rows to their owners like the
        // mma.sync consumers push their partials (slot [rank][0][m / cs] of owner m % cs)
        constexpr int NM = MT <= 2 ? 16 : 32;
        const int wq = warp & 3, row = wq * 32 + lane;
        const uint32_t dcol = uint32_t(4 * (BITS == 4 ? 64 : 32) + pbuf * NM);
        float d[NM];
        if (ok) ok = mbar_wait(&dfull[pbuf], uint32_t((j >> 1) & 1), p.status, kErrWaitMma);
        tcg::tc_fence_after();
        tcg::tmem_ld16(*tmem_slot + (uint32_t(wq * 32) << 16) + dcol, d);
        if (NM == 32) tcg::tmem_ld16(*tmem_slot + (uint32_t(wq * 32) << 16) + dcol + 16, d + 16);
        tcg::tmem_wait_ld();
        tcg::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dempty[pbuf]);
        if (j >= 2 && ok)
          ok = mbar_wait_cluster(&freeb[pbuf], ((j - 2) >> 1) & 1, p.status, kErrWaitCluster);
        const uint32_t pa = smem_u32(part + (pbuf * cs + rank) * 2 * ro * PSTR);
        const uint32_t rb = smem_u32(&ready[pbuf]);
#pragma unroll
        for (int m = 0; m < RP; ++m) {
          const int owner = m % cs, ml = m / cs;
          const uint32_t a = pa + uint32_t((ml * PSTR + row) * 4);
          if (owner == rank)
            asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(d[m]) : "memory");
          else
            st_async_f32(mapa_shared(a, owner), d[m], mapa_shared(rb, owner));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ready[pbuf]);  // this warp's local rows are in place
      }
      if (etid == 0) mbar_arrive_expect_tx(&ready[pbuf], peer_bytes);
      if (ok) ok = mbar_wait_cluster(&ready[pbuf], (j >> 1) & 1, p.status, kErrWaitCluster);
      // sum the partials of each owned row: the two k halves of each rank, then the ranks in
      // order (local shared memory)
      for (int idx = etid; idx < nmine * (TN / 4); idx += NE) {
        const int mi = idx / (TN / 4), n4 = idx - mi * (TN / 4);
        const int m = rank + mi * cs;
        float4 s;
        for (int c = 0; c < cs; ++c) {
          const float4 h0 = *reinterpret_cast<const float4*>(&pb[((c * 2) * ro + mi) * PSTR + n4 * 4]);
          const float4 h1 = TC ? make_float4(0.f, 0.f, 0.f, 0.f)
                               : *reinterpret_cast<const float4*>(&pb[((c * 2 + 1) * ro + mi) * PSTR + n4 * 4]);
          const float4 v = TC ? h0 : make_float4(h0.x + h1.x, h0.y + h1.y, h0.z + h1.z, h0.w + h1.w);
          if (c == 0) {
            s = v;
          } else {
            s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
          }
        }
        *reinterpret_cast<float4*>(&red[m * PSTR + n4 * 4]) = s;
      }
      asm volatile("bar.sync 2, %0;" ::"n"(NE));
      // every CTA may push its next partial into this buffer again (lane c -> CTA c); the last
      // two tiles' buffers are pushed into no more, and nobody waits for their release
      if (etid < cs && j + 2 < ntl) {
        if (cs > 1)
          mbar_arrive_cluster(&freeb[pbuf], etid);
        else
          mbar_arrive(&freeb[pbuf]);
      }
      if (!TC && cs > 1 && j + 3 == ntl) cluster_arrive();  // the exit barrier (see above)
      epilogue<EPI, TN, PSTR, PEER>(p, red, rank, cs, t, t * TN, NWE, WARP_EPI,
                                    EPI == EPI_RESID ? pre : nullptr, EPI == EPI_QKROPE, qk);
      asm volatile("bar.sync 2, %0;" ::"n"(NE));  // red reads done
      if (PEER && p.peer_world > 0 && nmine > 0) {
        // this tile's rows, written locally by the epilogue, go to every peer's arena as
        // 16-byte copies (rows of 64-128 bf16, 16-byte aligned), then the elements are counted
        // on the peers' counters (the consumers wait for M x columns per source)
        const int col0 = EPI == EPI_SWIGLU ? t * (TN / 2) : t * TN;
        const int cols = EPI == EPI_SWIGLU ? min(TN / 2, p.n_act - col0) : min(TN, p.N - col0);
        if (cols > 0) {
          const int c16 = cols / 8;  // 16-byte chunks per row
          for (int idx = etid; idx < nmine * c16; idx += NE) {
            const int mi = idx / c16, c = idx - mi * c16;
            const char* src = reinterpret_cast<const char*>(p.out + (size_t)(rank + mi * cs) * p.ldo + col0) + c * 16;
            const uint4 v = *reinterpret_cast<const uint4*>(src);
            for (int q = 0; q < p.peer_world; ++q)
              if (p.peer_delta[q] != 0)
                *reinterpret_cast<uint4*>(const_cast<char*>(src) + p.peer_delta[q]) = v;
          }
          asm volatile("bar.sync 2, %0;" ::"n"(NE));  // every copy precedes the release
          if (etid == 0) {
            __threadfence_system();
            for (int q = 0; q < p.peer_world; ++q)
              red_add_release_sys(reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(p.peer_flag) +
                                                              p.peer_delta[q]),
                                  uint32_t(nmine * cols));
          }
        }
      }
    }
  }

  // No CTA leaves while a peer may still write its partial tiles or arrive on its barriers. The
  // mma.sync engine's warps made this barrier's arrive after their last access to a peer's shared
  // memory (the producer after its set-up wait, the consumers after their last push, the
  // epilogue warps after their last buffer release), so the wait here does not add a cluster
  // round trip after the last epilogue. Every partial pushed into this CTA has landed before
  // its last reduction (the ready barrier counts the bytes).
  if (TC) {
    if (cs > 1) cluster_sync_all(); else __syncthreads();
  } else {
    if (cs > 1) cluster_wait(); else __syncthreads();
  }
  // a gather wait: the launch's last CTA advances this rank's cumulative target (every CTA read
  // it before counting itself here)
  if (PEER && p.wait_flag != nullptr && tid == 0) {
    __threadfence();
    const uint32_t nctas = gridDim.x * gridDim.y;
    if (atomicAdd(&p.wait_state[1], 1u) == nctas - 1) {
      p.wait_state[1] = 0;
      p.wait_state[0] += p.wait_elems;
      __threadfence();
    }
  }
  if constexpr (TC) {
    if (warp == 0) {
      tcg::tc_fence_after();
      tcg::tmem_dealloc(*tmem_slot, 512);
    }
  }
}

}  // namespace st

// ----------------------------------------------------------------------------- host side

int st_smem_bytes(int bits, int rt, int kslice, int nslots, int cs, bool tc) {
  // at least enough that one CTA fills an SM: CTAs never share an SM's tensor memory
  return std::max(st::layout(bits, rt, kslice, nslots, cs, tc).total, tc ? 120 * 1024 : 0);
}

template <typename Kern>
static cudaError_t configure_st(Kern kern) {
  int optin = 0;
  cudaError_t e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin,
                                         current_device());
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
}

// Clusters of `cs` CTAs (each requesting `smem` bytes) that the device runs at once.
int st_max_clusters(int cs, int smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int>, int> cache;
  const int dev = current_device();
  const auto key = std::make_tuple(dev, cs, smem);
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int n = sm_count(dev) / cs;
  // occupancy depends on the launch shape only; one instance answers for all
  auto kern = st::qmm_st_kernel<4, 2, EPI_PLAIN, false>;
  if (configure_st(kern) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cs, 1);
    cfg.blockDim = dim3(st::NTHR);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = cs;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int c = 0;
    if (cudaOccupancyMaxActiveClusters(&c, kern, &cfg) == cudaSuccess && c > 0) n = c;
  }
  cudaGetLastError();  // a refused query leaves the estimate; clear its error
  std::lock_guard<std::mutex> g(mu);
  cache[key] = n;
  return n;
}

template <int BITS, int MT, int EPI, bool TC, bool PEER = false>
static int launch_st(const QmmParams& p, const QmmPlan& pl, cudaStream_t stream) {
  auto kern = st::qmm_st_kernel<BITS, MT, EPI, TC, PEER>;
  const int smem = st_smem_bytes(BITS, MT, pl.kslice, pl.nslots, pl.cs, TC);
  DSPARK_CUDA_TRY(configure_once(reinterpret_cast<const void*>(kern), 1,
                                 [&] { return configure_st(kern); }),
                  "qmm_st: set smem / cluster attributes");
  CUtensorMap wmap, smap, bmap;
  if (!tma_maps(p, st::TN, true, &wmap, &smap, &bmap)) return DSPARK_ERR_CUDA;
  const int ntiles = (p.N + st::TN - 1) / st::TN;
  int nclus = pl.clusters > 0 ? pl.clusters : sm_count(current_device()) / pl.cs;
  nclus = std::max(1, std::min(nclus, ntiles));
  DSPARK_CUDA_TRY(launch_ex(kern, dim3(pl.cs, nclus), dim3(TC ? st::NTHR_TC : st::NTHR),
                            (size_t)smem, stream, pl.cs,
                            true, wmap, smap, bmap, p),
                  "qmm_st: launch");
  return DSPARK_OK;
}

template <int BITS, int EPI>
static int st_dispatch(const QmmParams& p, const QmmPlan& pl, cudaStream_t s) {
  if (pl.tcmma) {
    if (p.M <= 8) return launch_st<BITS, 1, EPI, true>(p, pl, s);
    if (p.M <= 16) return launch_st<BITS, 2, EPI, true>(p, pl, s);
    return launch_st<BITS, 4, EPI, true>(p, pl, s);
  }
  if (p.peer_world > 0 || p.wait_flag != nullptr) {  // the tensor-parallel instances
    if (p.M <= 8) return launch_st<BITS, 1, EPI, false, true>(p, pl, s);
    if (p.M <= 16) return launch_st<BITS, 2, EPI, false, true>(p, pl, s);
    return launch_st<BITS, 4, EPI, false, true>(p, pl, s);
  }
  if (p.M <= 8) return launch_st<BITS, 1, EPI, false>(p, pl, s);
  if (p.M <= 16) return launch_st<BITS, 2, EPI, false>(p, pl, s);
  return launch_st<BITS, 4, EPI, false>(p, pl, s);
}

int run_st(const QmmParams& p, int epi, const QmmPlan& pl, cudaStream_t s) {
  if (!pl.sct || p.K % st::KBLK)
    return fail(DSPARK_ERR_UNSUPPORTED, "qmm_st: needs K %% 512 == 0 and 16-byte aligned scales");
  if (pl.kslice % st::KBLK) return fail(DSPARK_ERR_ARG, "qmm_st: k slice %d", pl.kslice);
  if (pl.kslice / st::KBLK > st::kXBlocks)
    return fail(DSPARK_ERR_UNSUPPORTED, "qmm_st: k slice %d (at most %d)", pl.kslice,
                st::kXBlocks * st::KBLK);
  if (p.bits == 4) {
    switch (epi) {
      case EPI_PLAIN: return st_dispatch<4, EPI_PLAIN>(p, pl, s);
      case EPI_RESID: return st_dispatch<4, EPI_RESID>(p, pl, s);
      case EPI_SWIGLU: return st_dispatch<4, EPI_SWIGLU>(p, pl, s);
      case EPI_QKROPE: return st_dispatch<4, EPI_QKROPE>(p, pl, s);
    }
  } else {
    switch (epi) {
      case EPI_PLAIN: return st_dispatch<8, EPI_PLAIN>(p, pl, s);
      case EPI_RESID: return st_dispatch<8, EPI_RESID>(p, pl, s);
      case EPI_SWIGLU: return st_dispatch<8, EPI_SWIGLU>(p, pl, s);
      case EPI_QKROPE: return st_dispatch<8, EPI_QKROPE>(p, pl, s);
    }
  }
  return fail(DSPARK_ERR_ARG, "qmm_st: bad epilogue %d", epi);
}

}  // namespace qmm
}  // namespace dspark
