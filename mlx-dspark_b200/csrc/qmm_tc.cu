// K1 on the 5th-generation tensor cores: small-M affine-quantized matmul with tcgen05.mma
// (sm_100a). Same contract and numerics as qmm.cu (y[M,N] = x[M,K] . dequant(W)^T, MLX affine
// 4/8-bit group 64, fp32 accumulation, per-group scale/bias fold), different engine:
//
//  * Persistent clusters. The grid is (cs, P): cs CTAs per cluster split K into cs slices, and
//    P clusters (as many as fit on the GPU at once, never more than there are tiles) walk the
//    128-row output tiles t = cluster, cluster + P, ... Each CTA stages its K-slice of x once
//    and keeps it for every tile it visits; its producer warp streams the packed weights and
//    their scales/biases through a shared-memory ring with TMA without a break between tiles.
//  * Two consumer warpgroups alternate quantization groups. Thread t of a warpgroup owns weight
//    row t: it dequantizes its row's 64 weights of the group in registers with the bf16
//    magic-exponent trick (nibble | 0x4300 = 128 + q, exact) and writes them to tensor memory
//    with tcgen05.st — the MMA's A operand lives in TMEM (lane = row, two bf16 per column).
//  * x (the B operand, 16 or 32 rows) sits in shared memory in the UMMA canonical K-major
//    no-swizzle layout (8-row x 16-byte core matrices), with k permuted inside each 8-block
//    exactly as the magic extraction orders the weights.
//  * One thread per warpgroup issues tcgen05.mma (M=128, N=16|32, K=16) into a per-group fp32
//    accumulator in TMEM and commits to an mbarrier; the warpgroup reads the group's product P
//    back with tcgen05.ld and folds acc += scale*P + (bias - MAGIC*scale)*sum_k x in registers
//    while the tensor core works on the next group (accumulators double-buffered in TMEM).
//  * 8-bit weights are two exact 4-bit planes (lo: 128+lo, hi: 256+16*hi), two MMAs per k16.
//  * Split-K partial tiles are exchanged through distributed shared memory: each CTA publishes
//    its partial tile (double-buffered) and signals every peer's "ready" mbarrier; each CTA
//    sums its rows m = rank + i*cs over the cs partials in fixed rank order, signals "free",
//    and runs the shared epilogue on them.
// Every mbarrier wait is time-bounded (a failed wait records an error and the kernel drains
// without further waits on other agents); TMEM is always released before the CTA exits.
#include <algorithm>
#include <cmath>
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

namespace tc {

using namespace ::dspark::tcg;

constexpr int TN = 128;          // weight rows per tile (= MMA M)
constexpr int KSTG = 512;        // k per pipeline stage
constexpr int GPS = KSTG / 64;   // groups per stage
constexpr int NWG = 2;           // dequantizing warpgroups (and as many folding warpgroups)
constexpr int NX = 2 * NWG * 128;  // dequant + fold threads (they stage x together)
constexpr int NF = NWG * 128;      // fold threads (tile end: split-K exchange, epilogue)
constexpr int WARP_FOLD = NWG * 4;     // first fold warp
constexpr int WARP_MMA = 2 * NWG * 4;  // the warp that issues the tensor-core MMAs
constexpr int WARP_TMA = WARP_MMA + 1; // the producer warp
constexpr int NTHR = (WARP_TMA + 1) * 32;
constexpr int PSTR = TN + 4;
constexpr int MAXA = 4;          // A buffers per warpgroup, at most
constexpr int MAXD = 8;          // D buffers per warpgroup, at most

template <int BITS>
struct Tr;
template <>
struct Tr<4> {
  static constexpr float MAGIC = 128.0f;
  static constexpr int SB = 2;        // 128-byte boxes per stage row
  static constexpr int ACOLS = 32;    // TMEM columns of one group's A (64 k of bf16 pairs)
};
template <>
struct Tr<8> {
  static constexpr float MAGIC = 384.0f;  // 128 (low plane) + 256 (high plane)
  static constexpr int SB = 4;
  static constexpr int ACOLS = 64;    // low plane 32 + high plane 32
};

// Per warpgroup: A buffers (one group of dequantized weights each; the tensor core frees them
// within a few hundred cycles) and D buffers (one group's fp32 product each; the fold warps free
// them, and they must ride out the fold's work at the end of a tile), in half of TMEM.
// The roles hand over units of UG groups (two for 4-bit, one for 8-bit), so every barrier
// round trip is paid once per 4 KB of weights per row block.
__host__ __device__ constexpr int ugroups(int bits) { return bits == 4 ? 2 : 1; }
__host__ __device__ constexpr int nabuf(int bits) { return 2; }
__host__ __device__ constexpr int ndbuf(int bits, int nm) {
  return (256 - nabuf(bits) * ugroups(bits) * (bits == 4 ? 32 : 64)) / (ugroups(bits) * nm) < MAXD
             ? (256 - nabuf(bits) * ugroups(bits) * (bits == 4 ? 32 : 64)) / (ugroups(bits) * nm)
             : MAXD;
}

struct Layout {
  int ring, scs, bis, xs, sx, part, red, rs, bars, tmem, total;
};

__host__ __device__ inline int stage_bytes(int bits) {
  return (bits == 4 ? Tr<4>::SB : Tr<8>::SB) * TN * 128 + 2 * TN * 16;
}

__host__ __device__ inline Layout layout(int bits, int rt, int kslice, int nslots) {
  const int sb = bits == 4 ? Tr<4>::SB : Tr<8>::SB;
  const int rp = 8 * rt, nm = rt <= 2 ? 16 : 32;
  Layout L;
  int off = 0;
  L.ring = off;
  off += nslots * sb * TN * 128;
  L.scs = off;
  off += nslots * TN * 16;
  L.bis = off;
  off += nslots * TN * 16;
  L.xs = off;
  off += (kslice / 8) * nm * 16;
  L.sx = off;
  off += (kslice / 64) * rp * 4;
  off = (off + 15) & ~15;
  L.part = off;                 // two partial-tile buffers
  off += 2 * rp * PSTR * 4;
  L.red = off;
  off += rp * PSTR * 4;
  L.rs = off;
  off += 32 * 4;
  off = (off + 15) & ~15;
  L.bars = off;
  off += (2 * nslots + 2 * NWG * (MAXA + MAXD) + 4) * 8;
  L.tmem = off;
  off += 16;
  L.total = off + 1024;
  return L;
}

constexpr int kTmemCols = 512;  // every configuration allocates all of it (one CTA per SM)

// ------------------------------------------------------------------ kernel
//
// Warp roles (one CTA per SM, 576 threads):
//   warps 0..7   two dequantizing warpgroups: warpgroup w takes the units (UG groups) u = w,
//                w+2, ... of every stage and writes them to its A buffers in TMEM. After the
//                next tile's units they also finish a tile: split-K exchange and epilogue,
//                when the cluster peers have long published their partials
//   warps 8..15  two folding warpgroups: warpgroup w reads the products of warpgroup w's
//                units from its D buffers, folds them into per-row accumulators and at the
//                end of a tile publishes the CTA's partial tile
//   warp 16      issues the MMAs (warp-uniform, one elected lane) and commits them
//   warp 17      the TMA producer
// Per warpgroup w, group i of that warpgroup uses A buffer i % NA and D buffer i % ND:
//   afull[w][a]   4 dequant warps -> MMA warp   (A written)
//   adone[w][a]   tcgen05.commit  -> dequant    (A free again)
//   dfull[w][d]   tcgen05.commit  -> fold       (D ready)
//   dempty[w][d]  4 fold warps    -> MMA warp   (D read)

template <int BITS, int RT, int EPI, bool SCT>
__global__ void __launch_bounds__(NTHR, 1)
    qmm_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
                  const __grid_constant__ CUtensorMap bmap, const QmmParams p) {
  constexpr int RP = 8 * RT;                 // x rows that matter
  constexpr int NM = RT <= 2 ? 16 : 32;      // MMA N (x rows staged, zero padded)
  constexpr int SB = Tr<BITS>::SB;
  constexpr int BOX = TN * 128;
  constexpr int STG = SB * BOX;
  constexpr int SCB = TN * 16;
  constexpr int ACOLS = Tr<BITS>::ACOLS;
  constexpr float MAGIC = Tr<BITS>::MAGIC;
  constexpr uint32_t IDESC = idesc_bf16(NM);
  constexpr int UG = ugroups(BITS);
  constexpr int NA = nabuf(BITS);
  constexpr int ND = ndbuf(BITS, NM);
  constexpr int AU = UG * ACOLS;             // TMEM columns of one unit's A
  constexpr int DU = UG * NM;                // TMEM columns of one unit's D
  constexpr int PER = NA * AU + ND * DU;     // TMEM columns per warpgroup
  static_assert(NWG * PER <= kTmemCols && ND >= 2, "TMEM budget");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align_up<1024>(smem_raw);
  const int S = p.nslots;
  const Layout Lo = layout(BITS, RT, p.kslice, S);
  uint8_t* ring = smem + Lo.ring;
  uint8_t* scs = smem + Lo.scs;
  uint8_t* bis = smem + Lo.bis;
  uint8_t* xs = smem + Lo.xs;
  float* sx = reinterpret_cast<float*>(smem + Lo.sx);
  float* part = reinterpret_cast<float*>(smem + Lo.part);
  float* red = reinterpret_cast<float*>(smem + Lo.red);
  float* rsm = reinterpret_cast<float*>(smem + Lo.rs);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lo.bars);
  uint64_t* empty = full + S;
  uint64_t* afull = empty + S;               // [NWG][MAXA]
  uint64_t* adone = afull + NWG * MAXA;      // [NWG][MAXA]
  uint64_t* dfull = adone + NWG * MAXA;      // [NWG][MAXD]
  uint64_t* dempty = dfull + NWG * MAXD;     // [NWG][MAXD]
  uint64_t* ready = dempty + NWG * MAXD;     // [2] cluster: peers' partial tiles published
  uint64_t* freeb = ready + 2;               // [2] cluster: peers done reading our partial
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lo.tmem);

  const int cs = p.cs;
  const int rank = blockIdx.x;
  const int ntiles = (p.N + TN - 1) / TN;
  const int nclus = gridDim.y;
  const int ntl = int(blockIdx.y) < ntiles ? (ntiles - int(blockIdx.y) + nclus - 1) / nclus : 0;
  const int kbase = rank * p.kslice;
  const int kvalid = min(p.kslice, p.K - kbase);
  const int nst = (kvalid + KSTG - 1) / KSTG;
  const int gslice = p.kslice / 64;
  const int gfirst = kbase / 64;
  const int ngroups = (kvalid + 63) / 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  // groups of stage st: gl = st*GPS + gi for gi < ngs(st) (the last stage of a slice may be short)
  auto ngs = [&](int st) { return max(0, min(GPS, min(ngroups, p.G - gfirst) - st * GPS)); };

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 2 * NWG * 4);
    }
    for (int i = 0; i < NWG * MAXA; ++i) {
      mbar_init(&afull[i], 4);
      mbar_init(&adone[i], 1);
    }
    for (int i = 0; i < NWG * MAXD; ++i) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dempty[i], 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ready[i], cs);
      mbar_init(&freeb[i], cs);
    }
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  if (cs > 1) cluster_sync_all(); else __syncthreads();  // peers' barriers exist before use
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  if (warp == WARP_TMA) {
    // ------------------------------------------------------------- producer warp
    if (lane == 0) {
      prefetch_tmap(&wmap);
      if (SCT) {
        prefetch_tmap(&smap);
        prefetch_tmap(&bmap);
      }
      const uint64_t pol = l2_policy_evict_first();
      const uint32_t bytes = STG + (SCT ? 2 * SCB : 0);
      bool ok = true;
      int issued = 0;
      for (int j = 0; j < ntl && ok; ++j) {
        const int n0 = (int(blockIdx.y) + j * nclus) * TN;
        for (int st = 0; st < nst; ++st) {
          const int g = j * nst + st;
          const int slot = g % S;
          if (g >= S && !mbar_wait(&empty[slot], ((g / S) - 1) & 1, p.status, kErrWaitEmpty)) {
            ok = false;
            break;
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
          ++issued;
        }
      }
      // never leave the CTA with copies in flight: wait (bounded) for the last ones issued
      for (int g = max(0, issued - S); g < issued; ++g)
        mbar_wait(&full[g % S], (g / S) & 1, p.status, kErrWaitFull);
    }
    __syncwarp();
  } else if (warp == WARP_MMA) {
    // ------------------------------------------------------------- MMA warp
    static_assert(NWG == 2, "the MMA warp interleaves two warpgroups");
    const uint64_t bd0 = smem_desc(smem_u32(xs), NM * 16, 128);
    int cnt0 = 0, cnt1 = 0;  // groups issued per warpgroup (scalars: no local-memory array)
    for (int j = 0; j < ntl; ++j) {
      for (int st = 0; st < nst; ++st) {
        const int ng = ngs(st);
        const int nu = (ng + UG - 1) / UG;
        for (int uu = 0; uu < nu; ++uu) {
          const int w = uu & 1;
          const int i = w ? cnt1++ : cnt0++;
          const int a = i % NA, ua = i / NA;
          const int d = i % ND, ud = i / ND;
          mbar_wait(&afull[w * MAXA + a], ua & 1, p.status, kErrWaitMma);
          if (ud > 0) mbar_wait(&dempty[w * MAXD + d], (ud - 1) & 1, p.status, kErrWaitMma);
          tc_fence_after();
          const uint32_t ta = tmem + w * PER + a * AU;
          const uint32_t td = tmem + w * PER + NA * AU + d * DU;
          // group gl's x: 8 blocks of 8 k at (gl*8 + blk) * NM * 16 bytes (descriptor units of 16)
          const uint64_t bd = bd0 + uint64_t((st * GPS + uu * UG) * 8 * NM);
          const int nug = min(UG, ng - uu * UG);
          if (elect_one()) {
#pragma unroll
            for (int gg = 0; gg < UG; ++gg) {
              if (gg < nug) {
#pragma unroll
                for (int s = 0; s < 4; ++s) {  // four k16 steps = 8 TMEM columns of A each
                  const uint64_t b = bd + uint64_t((gg * 8 + 2 * s) * NM);
                  umma_ts(td + gg * NM, ta + gg * ACOLS + 8 * s, b, IDESC, s > 0 ? 1u : 0u);
                  if (BITS == 8) umma_ts(td + gg * NM, ta + gg * ACOLS + 32 + 8 * s, b, IDESC, 1u);
                }
              }
            }
            umma_commit(&adone[w * MAXA + a]);
            umma_commit(&dfull[w * MAXD + d]);
          }
          __syncwarp();
        }
      }
    }
  } else {
    // ------------------------------------------------------------- dequant + fold warpgroups
    pdl_wait();
    if (p.norm_w != nullptr) {
      for (int m = warp; m < RP; m += NX / 32) {
        float ss = 0.f;
        if (m < p.M)
          for (int e = lane; e < p.ssq_n; e += 32) ss += __ldcg(&p.ssq_in[e * p.ssq_stride + m]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) rsm[m] = m < p.M ? rsqrtf(ss / float(p.K) + p.eps) : 0.f;
      }
      asm volatile("bar.sync 2, %0;" ::"n"(NX));
    }
    // stage x once, in the UMMA K-major canonical layout: block j (8 k) of row m at
    // (j*NM + m)*16, k order (0,4,1,5,2,6,3,7) for 4-bit, (0,2,1,3) per half-block for 8-bit
    {
      const int blocks = p.kslice / 8;
      const int total = NM * blocks;
      constexpr int XB = 4;
      const bool nrm = p.norm_w != nullptr;
      for (int base = tid; base < total; base += NX * XB) {
        uint4 v[XB], w[XB];
#pragma unroll
        for (int u = 0; u < XB; ++u) {
          const int idx = base + u * NX;
          const int j = idx / NM, m = idx - j * NM;
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
          const int idx = base + u * NX;
          if (idx >= total) break;
          const int j = idx / NM, m = idx - j * NM;
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
          *reinterpret_cast<uint4*>(xs + (j * NM + m) * 16) = o;
        }
      }
      asm volatile("bar.sync 2, %0;" ::"n"(NX));
      for (int idx = tid; idx < RP * gslice; idx += NX) {
        const int g = idx / RP, m = idx - g * RP;
        float s = 0.f;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
          const uint4 q = *reinterpret_cast<const uint4*>(xs + ((g * 8 + b) * NM + m) * 16);
          s += (bf16_lo(q.x) + bf16_hi(q.x)) + (bf16_lo(q.y) + bf16_hi(q.y)) +
               (bf16_lo(q.z) + bf16_hi(q.z)) + (bf16_lo(q.w) + bf16_hi(q.w));
        }
        sx[g * RP + m] = s;
      }
      fence_proxy_async_smem();  // x becomes the tensor core's B operand (async proxy)
      asm volatile("bar.sync 2, %0;" ::"n"(NX));
    }

    const int row = tid & 127;                // weight row within the tile == TMEM lane
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    const uint32_t ring_a = smem_u32(ring);
    bool ok = true;  // false once a wait on another agent ran out: drain without waiting

    if (warp < WARP_FOLD) {
      // --------------------------------------------------------- dequantizing warpgroup w
      const int w = warp >> 2;
      const uint32_t tab = tmem + w * PER + lane_off;
      const int nmine = (p.M > rank) ? (p.M - rank + cs - 1) / cs : 0;
      // split-K exchange + epilogue of tile jj (its partial sits in part[jj & 1] of every CTA
      // of the cluster once ready[jj & 1] completed), run by the dequant warps one tile after
      // the fold warps published it
      auto finish = [&](int jj) {
        const int pbuf = jj & 1;
        float* pb = part + pbuf * RP * PSTR;
        const int t = int(blockIdx.y) + jj * nclus;
        if (ok) ok = mbar_wait_cluster(&ready[pbuf], (jj >> 1) & 1, p.status, kErrWaitCluster);
        const float* src = pb;
        if (cs > 1) {
          for (int idx = tid; idx < nmine * (TN / 4); idx += NF) {
            const int mi = idx / (TN / 4), n4 = idx - mi * (TN / 4);
            const int m = rank + mi * cs;
            const uint32_t a = smem_u32(&pb[m * PSTR + n4 * 4]);
            float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int c = 0; c < cs; ++c) {
              const float4 v = ld_dsmem_f4(mapa_shared(a, c));
              s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
            }
            *reinterpret_cast<float4*>(&red[m * PSTR + n4 * 4]) = s;
          }
          asm volatile("bar.sync 3, %0;" ::"n"(NF));
          if (tid == 0)
            for (int c = 0; c < cs; ++c) mbar_arrive_cluster(&freeb[pbuf], c);
          src = red;
        }
        epilogue<EPI, TN, PSTR>(p, src, rank, cs, t, t * TN, NF / 32, 0);
        asm volatile("bar.sync 3, %0;" ::"n"(NF));  // red (or part) reads done
        if (cs == 1 && tid == 0) mbar_arrive(&freeb[pbuf]);
      };
      int i = 0;
      for (int j = 0; j < ntl; ++j) {
        for (int st = 0; st < nst; ++st) {
          const int g = j * nst + st;
          const int slot = g % S;
          if (ok) ok = mbar_wait(&full[slot], (g / S) & 1, p.status, kErrWaitFull);
          const uint32_t wbase = ring_a + slot * STG;
          const int ng = ngs(st);
          const int nu = (ng + UG - 1) / UG;
#pragma unroll 1
          for (int uu = w; uu < nu; uu += NWG, ++i) {
            const int a = i % NA, ua = i / NA;
            // A buffer a is free once the MMAs of its previous use completed (the tensor core
            // always finishes: wait even after a failure)
            if (ua > 0) mbar_wait(&adone[w * MAXA + a], (ua - 1) & 1, p.status, kErrWaitMma);
            tc_fence_after();
#pragma unroll
            for (int gg = 0; gg < UG; ++gg) {
            const int gi = uu * UG + gg;
            if (gi >= ng) break;
            const uint32_t ta = tab + a * AU + gg * ACOLS;
            if (BITS == 4) {
              const int box = gi >> 2;
              const int c0 = (gi & 3) * 2;
              uint4 wv[2];
#pragma unroll
              for (int h = 0; h < 2; ++h)
                wv[h] = lds128(wbase + box * BOX + row * 128 + (((c0 + h) ^ (row & 7)) << 4));
              const uint32_t wd[8] = {wv[0].x, wv[0].y, wv[0].z, wv[0].w,
                                      wv[1].x, wv[1].y, wv[1].z, wv[1].w};
              // word 2q+h, nibbles e and e+4 -> column 8q + 4h + e
              uint32_t r[32];
#pragma unroll
              for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                  for (int e = 0; e < 4; ++e)
                    r[8 * q + 4 * h + e] =
                        lop3_and_or(wd[2 * q + h] >> (4 * e), 0x000F000Fu, 0x43004300u);
              tmem_st32(ta, r);
            } else {
              const int box = gi >> 1;
              const int c0 = (gi & 1) * 4;
              uint4 wv[4];
#pragma unroll
              for (int h = 0; h < 4; ++h)
                wv[h] = lds128(wbase + box * BOX + row * 128 + (((c0 + h) ^ (row & 7)) << 4));
              const uint32_t* wd = reinterpret_cast<const uint32_t*>(wv);
              // word 4q+h -> low columns 8q + 2h, +1 and high columns 32 + 8q + 2h, +1
              uint32_t lo[32], hi[32];
#pragma unroll
              for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                  const uint32_t x = wd[4 * q + h];
                  lo[8 * q + 2 * h] = lop3_and_or(x, 0x000F000Fu, 0x43004300u);
                  lo[8 * q + 2 * h + 1] = lop3_and_or(x >> 8, 0x000F000Fu, 0x43004300u);
                  hi[8 * q + 2 * h] = lop3_and_or(x >> 1, 0x00780078u, 0x43804380u);
                  hi[8 * q + 2 * h + 1] = lop3_and_or(x >> 9, 0x00780078u, 0x43804380u);
                }
              tmem_st32(ta, lo);
              tmem_st32(ta + 32, hi);
            }
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&afull[w * MAXA + a]);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[slot]);
        }
        if (j >= 1) finish(j - 1);
      }
      if (ntl >= 1) finish(ntl - 1);
    } else {
      // --------------------------------------------------------- folding warpgroup w
      const int w = (warp - WARP_FOLD) >> 2;
      const int ftid = tid - WARP_FOLD * 32;   // 0 .. NF-1
      const uint32_t tdb = tmem + w * PER + NA * AU + lane_off;
      float acc[RP];
      int i = 0;
      for (int j = 0; j < ntl; ++j) {
        const int n0 = (int(blockIdx.y) + j * nclus) * TN;
#pragma unroll
        for (int m = 0; m < RP; ++m) acc[m] = 0.f;
        for (int st = 0; st < nst; ++st) {
          const int g = j * nst + st;
          const int slot = g % S;
          if (ok) ok = mbar_wait(&full[slot], (g / S) & 1, p.status, kErrWaitFull);
          uint4 sc8, bi8;
          if (SCT) {
            sc8 = lds128(smem_u32(scs + slot * SCB + row * 16));
            bi8 = lds128(smem_u32(bis + slot * SCB + row * 16));
          }
          const int ng = ngs(st);
          const int nu = (ng + UG - 1) / UG;
#pragma unroll 1
          for (int uu = w; uu < nu; uu += NWG, ++i) {
            const int d = i % ND, ud = i / ND;
            // the tensor core always finishes (its operands are local): wait even after a failure
            mbar_wait(&dfull[w * MAXD + d], ud & 1, p.status, kErrWaitMma);
            tc_fence_after();
            const int nug = min(UG, ng - uu * UG);
#pragma unroll
            for (int gg = 0; gg < UG; ++gg) {
            const int gi = uu * UG + gg;
            const int gl = st * GPS + gi;
            float sa, ba;
            if (SCT) {
              // select by value: a runtime index into the uint4 would go through local memory
              const int wi = gi >> 1;
              const uint32_t ws = wi == 0 ? sc8.x : wi == 1 ? sc8.y : wi == 2 ? sc8.z : sc8.w;
              const uint32_t wb = wi == 0 ? bi8.x : wi == 1 ? bi8.y : wi == 2 ? bi8.z : bi8.w;
              sa = (gi & 1) ? bf16_hi(ws) : bf16_lo(ws);
              ba = (gi & 1) ? bf16_hi(wb) : bf16_lo(wb);
            } else {
              const int nn = min(n0 + row, p.N - 1);
              sa = bf2f(p.scales[(size_t)nn * p.G + gfirst + gl]);
              ba = bf2f(p.biases[(size_t)nn * p.G + gfirst + gl]);
            }
            const float ca = ba - MAGIC * sa;
            const float4* sxg = reinterpret_cast<const float4*>(sx + (gi < ng ? gl : 0) * RP);
            // the product in 16-column pieces (fewer live registers); D is released after the
            // unit's last piece is in registers
#pragma unroll
            for (int h = 0; h < NM / 16; ++h) {
              float dv[16];
              tmem_ld16(tdb + d * DU + gg * NM + 16 * h, dv);
              tmem_wait_ld();
              if (gg == UG - 1 && h == NM / 16 - 1) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&dempty[w * MAXD + d]);
              }
              if (gg < nug) {
#pragma unroll
                for (int e4 = 0; e4 < 4; ++e4) {
                  const int m0 = 16 * h + 4 * e4;
                  if (m0 < RP) {  // acc = fma(s, P, fma(c, sum x, acc)), two rows per instruction
                    const float4 xs4 = sxg[m0 / 4];
                    fma2(acc[m0 + 0], acc[m0 + 1], ca, ca, xs4.x, xs4.y);
                    fma2(acc[m0 + 2], acc[m0 + 3], ca, ca, xs4.z, xs4.w);
                    fma2(acc[m0 + 0], acc[m0 + 1], sa, sa, dv[4 * e4 + 0], dv[4 * e4 + 1]);
                    fma2(acc[m0 + 2], acc[m0 + 3], sa, sa, dv[4 * e4 + 2], dv[4 * e4 + 3]);
                  }
                }
              }
            }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[slot]);
        }

        // ---- partial tile -> part[j & 1] ([m][row]); the two warpgroups add in fixed order
        const int pbuf = j & 1;
        float* pb = part + pbuf * RP * PSTR;
        // part[pbuf] last held tile j-2: every CTA of the cluster (this one included) must be
        // done reading it
        if (j >= 2 && ok)
          ok = mbar_wait_cluster(&freeb[pbuf], ((j - 2) >> 1) & 1, p.status, kErrWaitCluster);
        if (w == 0) {
#pragma unroll
          for (int m = 0; m < RP; ++m) pb[m * PSTR + row] = acc[m];
        }
        asm volatile("bar.sync 1, %0;" ::"n"(NF));
        if (w == 1) {
#pragma unroll
          for (int m = 0; m < RP; ++m) pb[m * PSTR + row] += acc[m];
        }
        asm volatile("bar.sync 1, %0;" ::"n"(NF));
        if (ftid == 0) {  // publish to every CTA of the cluster
          if (cs > 1) {
            fence_acq_rel_cluster();
            for (int c = 0; c < cs; ++c) mbar_arrive_cluster(&ready[pbuf], c);
          } else {
            mbar_arrive(&ready[pbuf]);
          }
        }
      }
    }
  }
  tc_fence_before();

  // no CTA leaves while a peer may still read its partial tiles or arrive on its barriers
  // (and every MMA has completed: the fold warps waited for the last ones)
  if (cs > 1) cluster_sync_all(); else __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace tc

// ----------------------------------------------------------------------------- host side

int tc_smem_bytes(int bits, int rt, int kslice, int nslots) {
  return tc::layout(bits, rt, kslice, nslots).total;
}

// The dynamic shared memory a launch requests: at least enough that one CTA fills an SM, so
// CTAs never share an SM's tensor memory (a CTA blocked in tcgen05.alloc could otherwise wait on
// a co-resident CTA that waits on it through the cluster).
static int tc_launch_smem(int bits, int rt, int kslice, int nslots) {
  return std::max(tc::layout(bits, rt, kslice, nslots).total, 120 * 1024);
}

// Lets a kernel take up to the device's opt-in shared memory per block and clusters of 16.
// (The cap is the same for every launch, so a later launch with a larger ring never finds a
// smaller limit left by an earlier one.)
template <typename Kern>
static cudaError_t configure_tc(Kern kern) {
  int optin = 0;
  cudaError_t e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin,
                                         current_device());
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
}

template <int BITS, int RT, int EPI, bool SCT>
static int launch_tc(const QmmParams& p, const QmmPlan& pl, cudaStream_t stream) {
  auto kern = tc::qmm_tc_kernel<BITS, RT, EPI, SCT>;
  const int smem = tc_launch_smem(BITS, RT, pl.kslice, pl.nslots);
  DSPARK_CUDA_TRY(configure_once(reinterpret_cast<const void*>(kern), 1,
                                 [&] { return configure_tc(kern); }),
                  "qmm_tc: set smem / cluster attributes");
  CUtensorMap wmap, smap, bmap;
  if (!tma_maps(p, tc::TN, SCT, &wmap, &smap, &bmap)) return DSPARK_ERR_CUDA;
  const int ntiles = (p.N + tc::TN - 1) / tc::TN;
  int nclus = pl.clusters > 0 ? pl.clusters : sm_count(current_device()) / pl.cs;
  nclus = std::max(1, std::min(nclus, ntiles));
  dim3 grid(pl.cs, nclus);
  DSPARK_CUDA_TRY(launch_ex(kern, grid, dim3(tc::NTHR), (size_t)smem, stream, pl.cs, true, wmap,
                            smap, bmap, p),
                  "qmm_tc: launch");
  return DSPARK_OK;
}

// Clusters of `cs` CTAs (each requesting `smem` bytes) that the device runs at once.
int tc_max_clusters(int bits, int rt, int cs, int smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int>, int> cache;
  const int dev = current_device();
  const auto key = std::make_tuple(dev, bits, rt, cs, smem);
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const int sms = sm_count(dev);
  int n = sms / cs;
  auto query = [&](auto kern) {
    if (configure_tc(kern) != cudaSuccess) return;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cs, 1);
    cfg.blockDim = dim3(tc::NTHR);
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
  };
  // occupancy depends on the launch shape only; any instance of the kernel answers for all
  if (bits == 4) {
    if (rt <= 1) query(tc::qmm_tc_kernel<4, 1, EPI_PLAIN, true>);
    else if (rt <= 2) query(tc::qmm_tc_kernel<4, 2, EPI_PLAIN, true>);
    else query(tc::qmm_tc_kernel<4, 4, EPI_PLAIN, true>);
  } else {
    if (rt <= 1) query(tc::qmm_tc_kernel<8, 1, EPI_PLAIN, true>);
    else if (rt <= 2) query(tc::qmm_tc_kernel<8, 2, EPI_PLAIN, true>);
    else query(tc::qmm_tc_kernel<8, 4, EPI_PLAIN, true>);
  }
  cudaGetLastError();  // a refused query leaves the estimate; clear its error
  std::lock_guard<std::mutex> g(mu);
  cache[key] = n;
  return n;
}

int tc_stage_bytes(int bits) { return tc::stage_bytes(bits); }
int tc_planned_smem(int bits, int rt, int kslice, int nslots) {
  return tc_launch_smem(bits, rt, kslice, nslots);
}

template <int BITS, int EPI>
static int tc_dispatch(const QmmParams& p, const QmmPlan& pl, cudaStream_t s) {
  if (!pl.sct && EPI != EPI_PLAIN)
    return fail(DSPARK_ERR_UNSUPPORTED, "qmm: fused epilogues need K %% 512 == 0");
  if (p.M <= 8) return pl.sct ? launch_tc<BITS, 1, EPI, true>(p, pl, s) : launch_tc<BITS, 1, EPI, false>(p, pl, s);
  if (p.M <= 16) return pl.sct ? launch_tc<BITS, 2, EPI, true>(p, pl, s) : launch_tc<BITS, 2, EPI, false>(p, pl, s);
  return pl.sct ? launch_tc<BITS, 4, EPI, true>(p, pl, s) : launch_tc<BITS, 4, EPI, false>(p, pl, s);
}

int run_tc(const QmmParams& p, int epi, const QmmPlan& pl, cudaStream_t s) {
  if (p.bits == 4) {
    switch (epi) {
      case EPI_PLAIN: return tc_dispatch<4, EPI_PLAIN>(p, pl, s);
      case EPI_RESID: return tc_dispatch<4, EPI_RESID>(p, pl, s);
      case EPI_SWIGLU: return tc_dispatch<4, EPI_SWIGLU>(p, pl, s);
      case EPI_QKROPE: return tc_dispatch<4, EPI_QKROPE>(p, pl, s);
    }
  } else {
    switch (epi) {
      case EPI_PLAIN: return tc_dispatch<8, EPI_PLAIN>(p, pl, s);
      case EPI_RESID: return tc_dispatch<8, EPI_RESID>(p, pl, s);
      case EPI_SWIGLU: return tc_dispatch<8, EPI_SWIGLU>(p, pl, s);
      case EPI_QKROPE: return tc_dispatch<8, EPI_QKROPE>(p, pl, s);
    }
  }
  return fail(DSPARK_ERR_ARG, "qmm_tc: bad epilogue %d", epi);
}

}  // namespace qmm
}  // namespace dspark
