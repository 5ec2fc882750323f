// K1 on the 5th-generation tensor cores: small-M affine-quantized matmul with tcgen05.mma
// (sm_100a). Same contract and numerics as qmm.cu (y[M,N] = x[M,K] . dequant(W)^T, MLX affine
// 4/8-bit group 64, fp32 accumulation, per-group scale/bias fold), different engine:
//
//  * A CTA owns 128 weight rows (tile) x one split-K slice. A producer warp streams the packed
//    weights and their scales/biases through a shared-memory ring with TMA (as in qmm.cu).
//  * Two consumer warpgroups alternate quantization groups. Thread t of a warpgroup owns weight
//    row t: it dequantizes its row's 64 weights of the group in registers with the bf16
//    magic-exponent trick (nibble | 0x4300 = 128 + q, exact) and writes them to tensor memory
//    with tcgen05.st — the MMA's A operand lives in TMEM (lane = row, two bf16 per column).
//  * x (the B operand, 16 or 32 rows) is staged once per CTA in shared memory in the UMMA
//    canonical K-major no-swizzle layout (8-row x 16-byte core matrices), with k permuted inside
//    each 8-block exactly as the magic extraction orders the weights.
//  * One thread per warpgroup issues tcgen05.mma (M=128, N=16|32, K=16) into a per-group fp32
//    accumulator in TMEM and commits to an mbarrier; the warpgroup reads the group's product P
//    back with tcgen05.ld and folds acc += scale*P + (bias - MAGIC*scale)*sum_k x in registers
//    while the tensor core works on the next group (accumulators double-buffered in TMEM).
//  * 8-bit weights are two exact 4-bit planes (lo: 128+lo, hi: 256+16*hi), two MMAs per k16.
//  * Split-K across a thread-block cluster, reduced through distributed shared memory in fixed
//    rank order; epilogues shared with qmm.cu.
// Every mbarrier wait is time-bounded; TMEM is always released before the CTA exits.
#include <algorithm>

#include "common.cuh"
#include "host_common.h"
#include "qmm.h"
#include "qmm_epilogue.cuh"

namespace dspark {
namespace qmm {

namespace tc {

constexpr int TN = 128;          // weight rows per CTA (= MMA M)
constexpr int KSTG = 512;        // k per pipeline stage
constexpr int GPS = KSTG / 64;   // groups per stage
constexpr int NWG = 2;           // consumer warpgroups
constexpr int NTHR = NWG * 128 + 32;
constexpr int PSTR = TN + 4;

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

struct Layout {
  int ring, scs, bis, xs, sx, part, red, rs, bars, tmem, total;
};

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
  L.part = off;
  off += rp * PSTR * 4;
  L.red = off;
  off += rp * PSTR * 4;
  L.rs = off;
  off += 32 * 4;
  off = (off + 15) & ~15;
  L.bars = off;
  off += (2 * nslots + 2 * NWG) * 8;
  L.tmem = off;
  off += 16;
  L.total = off + 1024;
  return L;
}

__host__ __device__ inline int tmem_cols(int bits, int rt) {
  const int acols = bits == 4 ? Tr<4>::ACOLS : Tr<8>::ACOLS;
  const int nm = rt <= 2 ? 16 : 32;
  const int per_wg = 2 * acols + 2 * nm;
  const int need = NWG * per_wg;
  int c = 32;
  while (c < need) c <<= 1;
  return c;
}

// ------------------------------------------------------------------ tcgen05 helpers

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, int ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, int ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* d) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) d[i] = __uint_as_float(r[i]);
}

// D[tmem] (+)= A[tmem] . B[smem desc]^T, bf16 inputs, fp32 accumulate
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Shared-memory matrix descriptor: K-major, no swizzle, 8-row x 16-byte core matrices.
// lbo: bytes between the two 16-byte K chunks of one MMA; sbo: bytes between 8-row groups.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFF);
  d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFF) << 32;
  d |= uint64_t(1) << 46;  // descriptor version for sm_100
  return d;                // base offset 0, layout type 0 (no swizzle)
}

// kind::f16 instruction descriptor: bf16 A/B, fp32 D, K-major A and B, M=128, N=n.
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(128 >> 4) << 24);
}

// ------------------------------------------------------------------ kernel

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

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
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
  uint64_t* mmab = empty + S;                // [NWG][2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lo.tmem);

  const int cs = p.cs;
  const int rank = blockIdx.x;
  const int ntile = blockIdx.y;
  const int n0 = ntile * TN;
  const int kbase = rank * p.kslice;
  const int kvalid = min(p.kslice, p.K - kbase);
  const int nst = (kvalid + KSTG - 1) / KSTG;
  const int gslice = p.kslice / 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  constexpr int NC = NWG * 128;
  const int ncols = tmem_cols(BITS, RT);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NWG * 4);
    }
    for (int i = 0; i < 2 * NWG; ++i) mbar_init(&mmab[i], 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  if (warp == NWG * 4) {
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
    // ------------------------------------------------------------- consumer warpgroups
    pdl_wait();
    if (p.norm_w != nullptr) {
      for (int m = warp; m < RP; m += NWG * 4) {
        float ss = 0.f;
        if (m < p.M)
          for (int e = lane; e < p.ssq_n; e += 32) ss += __ldcg(&p.ssq_in[e * p.ssq_stride + m]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) rsm[m] = m < p.M ? rsqrtf(ss / float(p.K) + p.eps) : 0.f;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(NC));
    }
    // stage x in the UMMA K-major canonical layout: block j (8 k) of row m at (j*NM + m)*16,
    // k order (0,4,1,5,2,6,3,7) for 4-bit, (0,2,1,3) per half-block for 8-bit
    const int blocks = p.kslice / 8;
    const int total = NM * blocks;
    constexpr int XB = 8;
    const bool nrm = p.norm_w != nullptr;
    for (int base = tid; base < total; base += NC * XB) {
      uint4 v[XB], w[XB];
#pragma unroll
      for (int u = 0; u < XB; ++u) {
        const int idx = base + u * NC;
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
        const int idx = base + u * NC;
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
    asm volatile("bar.sync 1, %0;" ::"n"(NC));
    for (int idx = tid; idx < RP * gslice; idx += NC) {
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
    asm volatile("bar.sync 1, %0;" ::"n"(NC));

    const int wg = warp >> 2;                 // warpgroup
    const int row = tid & 127;                // weight row within the tile == TMEM lane
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    const uint32_t tm_a = tmem + wg * (2 * ACOLS + 2 * NM);   // this warpgroup's A buffers
    const uint32_t tm_d = tm_a + 2 * ACOLS;                   // and accumulators
    uint64_t* mb = mmab + wg * 2;
    const uint32_t xs_a = smem_u32(xs);
    const uint32_t ring_a = smem_u32(ring);
    const int gfirst = kbase / 64;
    const int ngroups = (kvalid + 63) / 64;

    float acc[RP];
#pragma unroll
    for (int m = 0; m < RP; ++m) acc[m] = 0.f;
    float pend_s = 0.f, pend_c = 0.f;  // scale / folded bias of the group in flight
    int pend_gl = -1, nissued = 0;

    auto fold_pending = [&]() {
      if (pend_gl < 0) return;
      const int b = (nissued - 1) & 1;
      mbar_wait(&mb[b], ((nissued - 1) >> 1) & 1, p.status, kErrWaitFull);
      tc_fence_after();
      float d[NM];
      tmem_ld16(tm_d + b * NM + lane_off, d);
      if (NM == 32) tmem_ld16(tm_d + b * NM + 16 + lane_off, d + 16);
      tmem_wait_ld();
      const float* sxg = sx + pend_gl * RP;
#pragma unroll
      for (int m = 0; m < RP; ++m) acc[m] = fmaf(pend_s, d[m], fmaf(pend_c, sxg[m], acc[m]));
      pend_gl = -1;
    };

    for (int st = 0; st < nst; ++st) {
      const int slot = st % S;
      mbar_wait(&full[slot], (st / S) & 1, p.status, kErrWaitFull);
      const uint32_t wbase = ring_a + slot * STG;
      uint4 sc8, bi8;
      if (SCT) {
        sc8 = lds128(smem_u32(scs + slot * SCB + row * 16));
        bi8 = lds128(smem_u32(bis + slot * SCB + row * 16));
      }
#pragma unroll 1
      for (int gi = wg; gi < GPS; gi += NWG) {
        const int gl = st * GPS + gi;
        if (gl >= ngroups || gfirst + gl >= p.G) break;
        // ---- dequantize this row's 64 weights of group gl into the A buffer
        const int abuf = nissued & 1;
        const uint32_t ta = tm_a + abuf * ACOLS + lane_off;
        if (BITS == 4) {
          const int box = gi >> 2;
          const int c0 = (gi & 3) * 2;
          uint4 wv[2];
#pragma unroll
          for (int h = 0; h < 2; ++h)
            wv[h] = lds128(wbase + box * BOX + row * 128 + (((c0 + h) ^ (row & 7)) << 4));
          const uint32_t wd[8] = {wv[0].x, wv[0].y, wv[0].z, wv[0].w, wv[1].x, wv[1].y, wv[1].z, wv[1].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {  // words 2q, 2q+1 -> columns 8q .. 8q+7
            uint32_t r[8];
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int i = 0; i < 4; ++i)
                r[4 * h + i] = lop3_and_or(wd[2 * q + h] >> (4 * i), 0x000F000Fu, 0x43004300u);
            tmem_st8(ta + 8 * q, r);
          }
        } else {
          const int box = gi >> 1;
          const int c0 = (gi & 1) * 4;
          uint4 wv[4];
#pragma unroll
          for (int h = 0; h < 4; ++h)
            wv[h] = lds128(wbase + box * BOX + row * 128 + (((c0 + h) ^ (row & 7)) << 4));
          const uint32_t* wd = reinterpret_cast<const uint32_t*>(wv);
#pragma unroll
          for (int q = 0; q < 4; ++q) {  // words 4q .. 4q+3 -> low columns 8q.., high 32+8q..
            uint32_t lo[8], hi[8];
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const uint32_t x = wd[4 * q + h];
              lo[2 * h] = lop3_and_or(x, 0x000F000Fu, 0x43004300u);
              lo[2 * h + 1] = lop3_and_or(x >> 8, 0x000F000Fu, 0x43004300u);
              hi[2 * h] = lop3_and_or(x >> 1, 0x00780078u, 0x43804380u);
              hi[2 * h + 1] = lop3_and_or(x >> 9, 0x00780078u, 0x43804380u);
            }
            tmem_st8(ta + 8 * q, lo);
            tmem_st8(ta + 32 + 8 * q, hi);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        asm volatile("bar.sync %0, 128;" ::"r"(2 + wg));
        // ---- one thread issues the group's MMAs, then commits to this buffer's barrier
        if (row == 0) {
          tc_fence_after();
          const uint32_t td = tm_d + abuf * NM;
          const uint32_t tab = tm_a + abuf * ACOLS;
#pragma unroll
          for (int s = 0; s < 4; ++s) {  // four k16 steps of the group
            const uint32_t xaddr = xs_a + (gl * 8 + 2 * s) * NM * 16;
            const uint64_t bd = smem_desc(xaddr, NM * 16, 128);
            // one k16 step = 8 TMEM columns of A (two bf16 per column)
            umma_ts(td, tab + 8 * s, bd, IDESC, s > 0 ? 1u : 0u);
            if (BITS == 8) umma_ts(td, tab + 32 + 8 * s, bd, IDESC, 1u);
          }
          umma_commit(&mb[abuf]);
        }
        __syncwarp();
        // ---- fold the previous group while this one runs on the tensor core
        fold_pending();
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
        pend_s = sa;
        pend_c = ba - MAGIC * sa;
        pend_gl = gl;
        ++nissued;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    fold_pending();
    // partial tile -> shared memory [m][row]; the two warpgroups add in fixed order
    if (wg == 0) {
#pragma unroll
      for (int m = 0; m < RP; ++m) part[m * PSTR + row] = acc[m];
    }
    asm volatile("bar.sync 1, %0;" ::"n"(NC));
    if (wg == 1) {
#pragma unroll
      for (int m = 0; m < RP; ++m) part[m * PSTR + row] += acc[m];
    }
    tc_fence_before();
  }

  // ------------------------------------------------------------- split-K reduction
  if (cs > 1) cluster_sync_all(); else __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
  const int nmine = (p.M > rank) ? (p.M - rank + cs - 1) / cs : 0;
  for (int idx = tid; idx < nmine * (TN / 4); idx += NTHR) {
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
  epilogue<EPI, TN, PSTR>(p, red, rank, cs, ntile, n0, NTHR / 32);
}

}  // namespace tc

// ----------------------------------------------------------------------------- host side

int tc_smem_bytes(int bits, int rt, int kslice, int nslots) {
  return tc::layout(bits, rt, kslice, nslots).total;
}

template <int BITS, int RT, int EPI, bool SCT>
static int launch_tc(const QmmParams& p, const QmmPlan& pl, cudaStream_t stream) {
  auto kern = tc::qmm_tc_kernel<BITS, RT, EPI, SCT>;
  // Every CTA allocates its TMEM columns up front and a cluster's CTAs wait on one another,
  // so the CTAs that can be resident on one SM must be able to hold their columns at the same
  // time (else a CTA blocked in tcgen05.alloc could wait on a peer that waits on it). Pad the
  // shared-memory request so at most 512 / ncols CTAs fit on an SM.
  const int ncols = tc::tmem_cols(BITS, RT);
  const int per_sm = 512 / ncols;
  const int smem_floor = per_sm >= 4 ? 0 : (228 * 1024) / (per_sm + 1) + 1024;
  const int smem = std::max(tc::layout(BITS, RT, pl.kslice, pl.nslots).total, smem_floor);
  static int configured = 0;
  if (smem > configured) {
    DSPARK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                    "qmm_tc: set smem");
    DSPARK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                    "qmm_tc: allow cluster 16");
    configured = smem;
  }
  CUtensorMap wmap, smap, bmap;
  if (!tma_maps(p, tc::TN, SCT, &wmap, &smap, &bmap)) return DSPARK_ERR_CUDA;
  dim3 grid(pl.cs, (p.N + tc::TN - 1) / tc::TN);
  DSPARK_CUDA_TRY(launch_ex(kern, grid, dim3(tc::NTHR), (size_t)smem, stream, pl.cs, true, wmap,
                            smap, bmap, p),
                  "qmm_tc: launch");
  return DSPARK_OK;
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
