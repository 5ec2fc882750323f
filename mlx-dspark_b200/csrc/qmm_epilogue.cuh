// Epilogues of the quantized matmul (both engines): applied to the split-K-reduced fp32 tile
// `red` ([rows][pstr], rows m = rank + i*cs of this cluster rank) of output columns
// n0 .. n0+TN-1.
#pragma once

#include "common.cuh"
#include "qmm.h"

namespace dspark {
namespace qmm {

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + __expf(-g)) * u; }

// Store v at addr and, in the peer-store instance (PEER), at the same offset in every rank's
// arena (p.peer_delta[s]; the own rank's delta is 0). Used for the scattered statistics words;
// the output rows reach the peers as 16-byte copies after the tile (qmm_st.cu).
template <bool PEER, typename T>
__device__ __forceinline__ void put(const QmmParams& p, T* addr, T v) {
  if (!PEER || p.peer_world == 0) {
    *addr = v;
    return;
  }
  for (int s = 0; s < p.peer_world; ++s)
    *reinterpret_cast<T*>(reinterpret_cast<char*>(addr) + p.peer_delta[s]) = v;
}

// Rows per warp of the prefetched residual epilogue (the streaming engine: 4 epilogue warps,
// at most 32 owned rows, so nwarps * kResidRows covers every row).
constexpr int kResidRows = 8;

// The residual words the EPI_RESID epilogue of tile n0 reads, loaded by the same threads ahead
// of the split-K reduction so that their latency overlaps the wait for the partial tiles (the
// residual comes from an earlier kernel).
template <int TN>
__device__ __forceinline__ void resid_prefetch(const QmmParams& p, int rank, int cs, int n0,
                                               int nwarps, int warp0, uint32_t (&pre)[2 * kResidRows]) {
  const int tidx = int(threadIdx.x) - warp0 * 32;
  const int warp = tidx >> 5, lane = tidx & 31;
  const int nmine = (p.M > rank) ? (p.M - rank + cs - 1) / cs : 0;
#pragma unroll
  for (int i = 0; i < kResidRows; ++i) {
    const int mi = warp + i * nwarps;
    const int m = rank + mi * cs;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int n = n0 + (lane + 32 * h) * 2;
      pre[i * 2 + h] = (mi < nmine && n < p.N)
                           ? __ldcg(reinterpret_cast<const unsigned int*>(p.resid + (size_t)m * p.ldr + n))
                           : 0u;
    }
  }
}

// What the EPI_QKROPE epilogue of a tile reads besides the tile: the q/k norm weights and RoPE
// frequencies of this lane's columns (the same for every row), and the cache position / slot
// offset of the warp's first row. Loaded ahead of the split-K reduction by the same threads, so
// that their latency overlaps the wait for the partial tiles.
struct QkPre {
  float nq[4], nk[4], f[2];
  int pos;
  int64_t kvo;
};

template <int TN>
__device__ __forceinline__ void qkrope_prefetch(const QmmParams& p, int rank, int cs, int nwarps,
                                                int warp0, QkPre& q) {
  constexpr int HPT = TN / 128;
  const int tidx = int(threadIdx.x) - warp0 * 32;
  const int warp = tidx >> 5, lane = tidx & 31;
  const int nmine = (p.M > rank) ? (p.M - rank + cs - 1) / cs : 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    q.nq[i] = bf2f(p.qnorm[lane + 32 * i]);
    q.nk[i] = bf2f(p.knorm[lane + 32 * i]);
  }
  q.f[0] = p.inv_freq[lane];
  q.f[1] = p.inv_freq[lane + 32];
  const int mi = warp / HPT;  // the warp's first item is u = warp
  const int m = rank + mi * cs;
  q.pos = mi < nmine ? p.row_pos[m] : 0;
  q.kvo = (mi < nmine && p.row_kv != nullptr) ? p.row_kv[m] : 0;
}

// Run by `nwarps` warps starting at warp `warp0` of the CTA. `pre`: the residual words from
// resid_prefetch for this tile (EPI_RESID, 128-column tiles), or null to load them here.
template <int EPI, int TN, int PSTR, bool PEER = false>
__device__ __forceinline__ void epilogue(const QmmParams& p, const float* red, int rank, int cs,
                                         int ntile, int n0, int nwarps, int warp0 = 0,
                                         const uint32_t* pre = nullptr, bool has_qk = false,
                                         QkPre qk = {}) {
  const int nthr = nwarps * 32;
  const int tidx = int(threadIdx.x) - warp0 * 32;
  const int warp = tidx >> 5, lane = tidx & 31;
  const int nmine = (p.M > rank) ? (p.M - rank + cs - 1) / cs : 0;  // rows m = rank + i*cs
  if constexpr (EPI == EPI_PLAIN) {
    for (int idx = tidx; idx < nmine * (TN / 2); idx += nthr) {
      const int mi = idx / (TN / 2), n2 = idx - mi * (TN / 2);
      const int m = rank + mi * cs;
      const int n = n0 + n2 * 2;
      if (n >= p.N) continue;
      float v0 = round_bf16(red[m * PSTR + n2 * 2]);
      float v1 = round_bf16(red[m * PSTR + n2 * 2 + 1]);
      if (p.bias != nullptr) {
        v0 += bf2f(p.bias[n]);
        v1 += bf2f(p.bias[n + 1]);
      }
      *reinterpret_cast<uint32_t*>(p.out + (size_t)m * p.ldo + n) = pack_bf16x2(v0, v1);
    }
  } else if constexpr (EPI == EPI_RESID) {
    // out = bf16(bf16(acc) + resid); ssq_out[ntile][m] = sum over the tile of out^2
    if (pre != nullptr && TN == 128) {
      // the resid_prefetch map: warp w takes rows mi = w, w + nwarps, ... (at most kResidRows
      // per warp), lane l columns 2l and 2l + 64 of the tile
#pragma unroll
      for (int i = 0; i < kResidRows; ++i) {
        const int mi = warp + i * nwarps;
        if (mi >= nmine) break;
        const int m = rank + mi * cs;
        float ss = 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int n2 = lane + 32 * h;
          const int n = n0 + n2 * 2;
          if (n >= p.N) continue;
          const uint32_t rr = pre[i * 2 + h];
          const float h0 = round_bf16(round_bf16(red[m * PSTR + n2 * 2]) + bf16_lo(rr));
          const float h1 = round_bf16(round_bf16(red[m * PSTR + n2 * 2 + 1]) + bf16_hi(rr));
          *reinterpret_cast<uint32_t*>(p.out + (size_t)m * p.ldo + n) = pack_bf16x2(h0, h1);
          ss += h0 * h0 + h1 * h1;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0 && p.ssq_out != nullptr) put<PEER>(p, &p.ssq_out[ntile * p.ssq_stride + m], ss);
      }
      return;
    }
    for (int mi = warp; mi < nmine; mi += nwarps) {
      const int m = rank + mi * cs;
      float ss = 0.f;
      for (int n2 = lane; n2 < TN / 2; n2 += 32) {
        const int n = n0 + n2 * 2;
        if (n >= p.N) continue;
        const uint32_t rr =
            __ldcg(reinterpret_cast<const unsigned int*>(p.resid + (size_t)m * p.ldr + n));
        const float h0 = round_bf16(round_bf16(red[m * PSTR + n2 * 2]) + bf16_lo(rr));
        const float h1 = round_bf16(round_bf16(red[m * PSTR + n2 * 2 + 1]) + bf16_hi(rr));
        *reinterpret_cast<uint32_t*>(p.out + (size_t)m * p.ldo + n) = pack_bf16x2(h0, h1);
        ss += h0 * h0 + h1 * h1;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0 && p.ssq_out != nullptr) put<PEER>(p, &p.ssq_out[ntile * p.ssq_stride + m], ss);
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    // tile rows: pairs of (32 gate rows, 32 up rows); act column = pair*32 + j
    constexpr int PAIRS = TN / 64;
    for (int idx = tidx; idx < nmine * PAIRS * 32; idx += nthr) {
      const int mi = idx / (PAIRS * 32), rem = idx - mi * (PAIRS * 32);
      const int pr = rem >> 5, j = rem & 31;
      const int m = rank + mi * cs;
      const int a = (ntile * PAIRS + pr) * 32 + j;
      if (a >= p.n_act) continue;
      const float g = round_bf16(red[m * PSTR + pr * 64 + j]);
      const float u = round_bf16(red[m * PSTR + pr * 64 + 32 + j]);
      p.out[(size_t)m * p.ldo + a] = __float2bfloat16_rn(silu_mul(g, u));
    }
  } else if constexpr (EPI == EPI_QKROPE) {
    // tile = TN/128 heads of 128; columns [q heads | k heads | v heads]
    constexpr int HPT = TN / 128;
    for (int u = warp; u < nmine * HPT; u += nwarps) {
      const int mi = u / HPT, t = u - mi * HPT;
      const int m = rank + mi * cs;
      const int hh = n0 / 128 + t;
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = round_bf16(red[m * PSTR + t * 128 + lane + 32 * i]);
      const bool first = has_qk && u == warp;
      const int pos = first ? qk.pos : p.row_pos[m];
      const int64_t kvo = first ? qk.kvo : (p.row_kv != nullptr ? p.row_kv[m] : 0);
      if (hh >= p.hq && (pos < 0 || pos >= p.kv_cap)) {  // never write past a cache slot
        if (lane == 0) report_error(p.status, 0x301);
        continue;
      }
      if (hh < p.hq + p.hk) {
        const bool isq = hh < p.hq;
        const bf16* nw = isq ? p.qnorm : p.knorm;
        float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float r = rsqrtf(ss / 128.0f + p.eps);
        float y[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          y[i] = round_bf16(v[i] * r *
                            (has_qk ? (isq ? qk.nq[i] : qk.nk[i]) : bf2f(nw[lane + 32 * i])));
        // rotate-half RoPE: pairs (d, d+64) for d = lane, lane+32
        float o[4];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float f = has_qk ? qk.f[i] : p.inv_freq[lane + 32 * i];
          float sn, c;
          sincosf(float(pos) * f, &sn, &c);
          o[i] = y[i] * c - y[i + 2] * sn;
          o[i + 2] = y[i] * sn + y[i + 2] * c;
        }
        if (isq) {
          bf16* dst = p.qout + (size_t)m * p.ldq + hh * 128;
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = __float2bfloat16_rn(o[i]);
        } else {
          bf16* dst = p.kcache + kvo + (int64_t)(hh - p.hq) * p.k_sh + (int64_t)pos * p.k_ss;
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = __float2bfloat16_rn(o[i]);
        }
      } else if (hh < p.hq + 2 * p.hk) {
        bf16* dst = p.vcache + kvo + (int64_t)(hh - p.hq - p.hk) * p.v_sh + (int64_t)pos * p.v_ss;
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = __float2bfloat16_rn(v[i]);
      }
    }
  }
}

}  // namespace qmm
}  // namespace dspark
