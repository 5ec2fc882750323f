// K2: multi-row causal GQA verify attention  (sm_100a)
//
// Replaces multirow_sdpa / _P1 / _P2 (src/mlx_dspark/multirow_attn.py:223-259, :52-178),
// the kernel behind mx.fast.scaled_dot_product_attention for few-row verify blocks.
//
// Semantics (multirow_attn.py:85-87, :120-124): all G*qL query rows of a KV head are packed
// (GQA head major, then q position), so each K/V byte is read once per head for all rows.
// Row qi of a block of qL rows over L keys sees keys <= L - qL + qi (causal) or all keys;
// the tree-verify variant (multirow_attn.py:184-195) sees every prefix key and, among the
// last qL keys, key L-qL+j iff bit j of anc[qi] is set. Softmax in fp32 (exp2 domain, scale
// folded in); P is rounded to bf16 for the P.V product, as in the reference.
//
// B200 design: one CTA per (key split, batch row, KV head, row group). A producer warp
// streams 64-key K/V tiles into a 3-slot shared-memory ring of padded rows with 16-byte
// cp.async copies (coalesced across lanes; any 16-byte-aligned row stride, so strided cache
// views need no copy; keys past the end zero-filled), completing on mbarriers. (Bulk copies
// of single 256-byte rows measured ~1.3 TB/s device-wide on B200: too small per request.)
// Consumer warps run Q.K^T and P.V on tensor cores (mma.m16n8k16, ldmatrix from padded
// rows) with a flash-attention online softmax; warps that split a tile's keys merge in shared
// memory, the key splits of a cluster merge through distributed shared memory, and (only
// when more splits are needed than a cluster holds) cluster groups merge through a workspace.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include <cuda_fp16.h>

#include "attn.h"
#include "common.cuh"
#include "host_common.h"

namespace dspark {
namespace attn {

constexpr int KT = 64;     // keys per stage (head_dim <= 128)
constexpr int NSLOT = 3;   // ring depth

// keys per stage: 32 for head_dim 256, so that the three-slot ring of padded K/V rows fits
__host__ __device__ constexpr int ktile(int d) { return d > 128 ? 32 : KT; }

// bf16 (or, with F16, fp16) tensor-core MMA D[16x8] += A[16x16] B[16x8] with fp32 accumulation
template <bool F16>
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (F16) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    mma_bf16_16816(c, a0, a1, a2, a3, b0, b1);
  }
}

// two fp32 values rounded to the input type (bf16 or fp16) and packed low-first
template <bool F16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (F16) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    return pack_bf16x2(lo, hi);
  }
}

// Workspace row of one partial: D accumulators, then m and l, padded to 16 bytes so the
// accumulators are written with aligned 16-byte stores.
template <int D>
constexpr int kWsRow = D + 4;

template <int D>
struct AttnSmem {
  static constexpr int ROWB = D * 2 + 16;           // padded row (bank-conflict-free ldmatrix)
  static constexpr int STG = 2 * ktile(D) * ROWB;    // K tile + V tile
  static constexpr int RING = NSLOT * STG;
};

template <int D, int NRT, int KS>
__host__ __device__ constexpr int attn_core_bytes() {
  // ring (reused after the key loop for the merge buffers) + merge stats + barriers
  constexpr int RPG = NRT * 16;
  constexpr int merge = KS * RPG * D * 4;
  constexpr int ring = AttnSmem<D>::RING;
  constexpr int body = ring > merge ? ring : merge;
  return body + (2 * KS + 2) * RPG * 4 + 2 * NSLOT * 8 + 128;
}

// Receive area of the cluster merge: split s of a cluster pushes row r (owned by CTA r % ns)
// into slot [s][r / ns] of the owner, D accumulators then m and l (rows of D + 4 floats).
// Sized for any ns <= 16: ns * ceil(RPG / ns) <= RPG + 15 rows.
template <int D, int NRT>
__host__ __device__ constexpr int attn_recv_bytes() {
  return (NRT * 16 + 16) * (D + 4) * 4;
}

// + 1 KB: the base is aligned to 1024 bytes in the kernel (128-byte swizzled TMA destinations)
template <int D, int NRT, int KS>
__host__ __device__ constexpr int attn_smem_bytes() {
  return attn_core_bytes<D, NRT, KS>() + attn_recv_bytes<D, NRT>() + 1024;
}

// Byte offset of (key, d) inside a K or V tile. The cp.async ring keeps padded rows of ROWB
// bytes; the TMA ring (TM) keeps D/64 boxes of [KTD keys x 128 bytes] with the 128-byte swizzle
// (16-byte chunk c of a row r stored at chunk c ^ (r & 7)), so the 8 rows one ldmatrix phase
// reads always sit on 8 different bank groups. d is a multiple of 8.
template <bool TM, int KTD, int ROWB>
__device__ __forceinline__ uint32_t kv_off_in_tile(int key, int d) {
  if constexpr (TM)
    return uint32_t((d >> 6) * (KTD * 128) + key * 128 + ((((d >> 3) & 7) ^ (key & 7)) << 4));
  else
    return uint32_t(key * ROWB + d * 2);
}

// 2^x by the hardware approximation (ex2.approx.ftz: ~2 ulp; exact 0 for -inf)
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ int64_t q_base(const AttnParams& p, int b, const int64_t sb,
                                          const int64_t si) {
  return p.row_start ? int64_t(p.row_start[b]) * si : int64_t(b) * sb;
}

// DS warps share each (row tile, key slot): all of them compute the scores over the whole
// head_dim and each keeps D / DS output columns (DS = 2 for head_dim 256 bounds the registers).
// F16: fp16 inputs and output (the MMA type and the rounding of P follow the input type).
// QB (4 or 8): the K/V cache is MLX-affine quantized (p.kq / p.vq codes, bf16 scales / biases);
// four producer warps load the codes with 16-byte loads, dequantize (scale * q + bias, rounded to
// bf16) into the same padded ring rows, and arrive on the stage's barrier.
template <int QB>
__host__ __device__ constexpr int n_producers() { return QB ? 4 : 2; }

// TM: K/V tiles arrive by 2-D tensor-map copies (*kmap / *vmap over [.., L, D], no multicast)
// issued by one producer thread, instead of the producer warp's 16-byte cp.async copies. The
// body is shared by two entry points, so the default (cp.async) launch carries no tensor maps.
template <int D, int NRT, int KS, int DS, bool F16, int QB, bool TM>
__device__ __forceinline__ void attn_body(const CUtensorMap* kmap, const CUtensorMap* vmap,
                                          const AttnParams& p) {
  constexpr int NC = NRT * KS * DS;
  constexpr int NP = n_producers<QB>();
  constexpr int RPG = NRT * 16;
  constexpr int ROWB = AttnSmem<D>::ROWB;
  constexpr int STG = AttnSmem<D>::STG;
  constexpr int KTD = ktile(D);        // keys per stage
  constexpr int KPW = KTD / KS;        // keys per warp per stage (64 or 32)
  constexpr int KB = 32;               // keys per softmax step
  static_assert(KPW % KB == 0, "key slots of whole softmax steps");
  constexpr int DW = D / DS;           // output columns per warp
  constexpr int NDT = DW / 8;          // n8 tiles of the warp's output
  constexpr int NKK = D / 16;          // k16 steps of Q.K^T

  extern __shared__ __align__(128) uint8_t smem_raw[];
  // the 128-byte swizzled TMA destinations need 1024-byte alignment (the allocation has 1 KB of
  // slack); the cp.async layout keeps the base as it is
  uint8_t* smem = TM ? smem_align_up<1024>(smem_raw) : smem_raw;
  uint8_t* ring = smem;
  constexpr int BODY = attn_core_bytes<D, NRT, KS>() - (2 * KS + 2) * RPG * 4 - 2 * NSLOT * 8 - 128;
  float* bufO = reinterpret_cast<float*>(smem);            // [KS][RPG][D] (aliases the ring)
  float* bufM = reinterpret_cast<float*>(smem + BODY);     // [KS][RPG]
  float* bufL = bufM + KS * RPG;                           // [KS][RPG]
  float* finM = bufL + KS * RPG;                           // [RPG]
  float* finL = finM + RPG;                                // [RPG]
  uint64_t* full = reinterpret_cast<uint64_t*>(finL + RPG);
  uint64_t* empty = full + NSLOT;
  float* recv = reinterpret_cast<float*>(smem + attn_core_bytes<D, NRT, KS>());

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sidx_c = blockIdx.x;                 // split within the cluster
  const int g_grp = blockIdx.z;                  // cluster group
  const int bhr = blockIdx.y;                    // (b * Hk + hk) * nrg + rg
  const int rg = bhr % p.nrg;
  const int bh = bhr / p.nrg;
  const int hk = bh % p.Hk;
  const int b = bh / p.Hk;
  const int G = p.Hq / p.Hk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(&full[s], TM ? 1 : 32 * NP);  // the TMA thread's expect-tx, or every producer lane
      mbar_init(&empty[s], NC);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  pdl_wait();  // q and the freshly appended cache rows come from the previous kernel

  // The request's scalars (keys, query rows, cache offset, first packed row). When they come
  // from device arrays, one thread reads them and shares them through shared memory: every CTA
  // of the launch reads the same words at the same moment, and one request per CTA instead of
  // one per warp keeps their L2 line from queueing (the four loads issue together).
  int64_t* scal = reinterpret_cast<int64_t*>(empty + NSLOT);  // in the layout's 128-byte tail
  const bool dev_scalars = p.kv_len || p.q_len || p.kv_off || p.row_start;
  if (dev_scalars) {
    if (threadIdx.x == 0) {
      const int lb = p.kv_len ? p.kv_len[b] : p.L;
      const int ql = p.q_len ? p.q_len[b] : p.qL;
      const int64_t ko = p.kv_off ? p.kv_off[b] : 0;
      const int rs = p.row_start ? p.row_start[b] : 0;
      scal[0] = lb;
      scal[1] = ql;
      scal[2] = ko;
      scal[3] = rs;
    }
    __syncthreads();
  }
  const int Lb = dev_scalars ? int(scal[0]) : p.L;
  const int qLb = dev_scalars ? int(scal[1]) : p.qL;
  // q_base of this request: packed rows (row_start) or batch strides
  auto qbase = [&](int64_t sb, int64_t si) {
    return p.row_start ? scal[3] * si : int64_t(b) * sb;
  };
  const int split = g_grp * p.ns + sidx_c;
  const int k0 = min(Lb, split * p.chunk);
  const int kend = min(Lb, k0 + p.chunk);
  const int nst = (kend - k0 + KTD - 1) / KTD;

  const bf16* kb_ptr = p.k + (p.kv_off ? scal[2] : int64_t(b) * p.k_sb) + int64_t(hk) * p.k_sh;
  const bf16* vb_ptr = p.v + (p.kv_off ? scal[2] : int64_t(b) * p.v_sb) + int64_t(hk) * p.v_sh;

  if (QB != 0 && warp >= NC) {
    // ------------------------------------------------------------------ quantized producers
    constexpr int NPT = NP * 32;
    constexpr int QBE = QB ? QB : 8;           // (the branch is compiled, dead, for QB = 0)
    constexpr int CPR = D * QBE / 8 / 16;      // 16-byte code chunks per row
    constexpr int VPC = 128 / QBE;             // values per chunk (16 or 32)
    constexpr int NCH = 2 * KTD * CPR;         // chunks per stage, K then V
    constexpr int PER = NCH / NPT;             // chunks per producer thread per stage
    static_assert(NCH % NPT == 0, "whole chunks per producer thread");
    const int pt = (warp - NC) * 32 + lane;
    const uint32_t* kqp = p.kq + int64_t(b) * p.kq_sb + int64_t(hk) * p.kq_sh;
    const uint32_t* vqp = p.vq + int64_t(b) * p.kq_sb + int64_t(hk) * p.kq_sh;
    const int64_t sofs = int64_t(b) * p.ks_sb + int64_t(hk) * p.ks_sh;
    bool ok = true;
    for (int st = 0; st < nst && ok; ++st) {
      const int slot = st % NSLOT;
      if (st >= NSLOT) ok = mbar_wait(&empty[slot], ((st / NSLOT) - 1) & 1, p.status, kErrWaitKVEmpty);
      if (!ok) break;
      const int kt = k0 + st * KTD;
      constexpr int BATCH = PER < 4 ? PER : 4;  // chunks in flight per thread
#pragma unroll
      for (int i0 = 0; i0 < PER; i0 += BATCH) {
        uint4 pk[BATCH];
        float sc[BATCH], bi[BATCH];
#pragma unroll
        for (int i = 0; i < BATCH; ++i) {
          const int c = pt + (i0 + i) * NPT;
          const int kv = c / (KTD * CPR), rem = c - kv * (KTD * CPR);
          const int row = rem / CPR, ch = rem - row * CPR;
          const int key = kt + row;
          const bool valid = key < kend;
          const uint32_t* qb = (kv ? vqp : kqp) + int64_t(key) * p.kq_ss;
          pk[i] = valid ? ldg_v4(qb + ch * 4) : make_uint4(0u, 0u, 0u, 0u);
          const int64_t so = sofs + int64_t(key) * p.ks_ss + (ch * VPC) / 64;
          sc[i] = valid ? bf2f((kv ? p.vsc : p.ksc)[so]) : 0.f;
          bi[i] = valid ? bf2f((kv ? p.vbi : p.kbi)[so]) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < BATCH; ++i) {
          const int c = pt + (i0 + i) * NPT;
          const int kv = c / (KTD * CPR), rem = c - kv * (KTD * CPR);
          const int row = rem / CPR, ch = rem - row * CPR;
          uint8_t* dst = ring + slot * STG + kv * KTD * ROWB + row * ROWB + ch * VPC * 2;
          const uint32_t w[4] = {pk[i].x, pk[i].y, pk[i].z, pk[i].w};
#pragma unroll
          for (int e8 = 0; e8 < VPC / 8; ++e8) {
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              // values 2e', 2e' + 1 of the chunk, e' = 4 e8 + e. A code c becomes the float
              // 2^23 + c by placing it in the mantissa of 0x4B000000 (one byte permute for 8-bit
              // codes, a shift and a mask for 4-bit), minus 2^23 exactly: no int->float convert.
              constexpr int PERW = 32 / QBE;               // values per word
              const int v0 = 2 * (4 * e8 + e), v1 = v0 + 1;
              uint32_t m0, m1;
              if (QBE == 8) {
                m0 = __byte_perm(w[v0 / PERW], 0x4B000000u, 0x7540u + (v0 % PERW));
                m1 = __byte_perm(w[v1 / PERW], 0x4B000000u, 0x7540u + (v1 % PERW));
              } else {
                m0 = lop3_and_or(w[v0 / PERW] >> ((v0 % PERW) * 4), 0xFu, 0x4B000000u);
                m1 = lop3_and_or(w[v1 / PERW] >> ((v1 % PERW) * 4), 0xFu, 0x4B000000u);
              }
              const float f0 = __uint_as_float(m0) - 8388608.0f;
              const float f1 = __uint_as_float(m1) - 8388608.0f;
              o[e] = pack_bf16x2(fmaf(sc[i], f0, bi[i]), fmaf(sc[i], f1, bi[i]));
            }
            *reinterpret_cast<uint4*>(dst + 16 * e8) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
      }
      mbar_arrive(&full[slot]);
    }
  } else if (TM && warp == NC) {
    // ------------------------------------------------------------------ TMA producer thread
    // Per stage, D/64 boxes of [KTD keys x 64 dims] for K and the same for V, all on
    // full[slot]. Keys past the tensor's L are zero-filled by the copy; keys in [kend, L) are
    // real cache rows, masked in the scores and zeroed in the consumers' V fragments.
    if (lane == 0) {
      uint8_t* const ring0 = ring;
      bool ok = true;
      for (int st = 0; st < nst && ok; ++st) {
        const int slot = st % NSLOT;
        if (st >= NSLOT) ok = mbar_wait(&empty[slot], ((st / NSLOT) - 1) & 1, p.status, kErrWaitKVEmpty);
        if (!ok) break;
        const int kt = k0 + st * KTD;
        uint8_t* kd = ring0 + slot * STG;
        uint8_t* vd = kd + KTD * D * 2;
        mbar_arrive_expect_tx(&full[slot], uint32_t(2 * KTD * D * 2));
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx) {
          tma_load_4d(kd + bx * KTD * 128, kmap, &full[slot], bx * 64, kt, hk, b);
          tma_load_4d(vd + bx * KTD * 128, vmap, &full[slot], bx * 64, kt, hk, b);
        }
      }
      // never leave with copies in flight: wait (bounded) for the last stages issued
      for (int st = max(0, nst - NSLOT); st < nst && ok; ++st)
        mbar_wait(&full[st % NSLOT], (st / NSLOT) & 1, p.status, kErrWaitKV);
    }
    __syncwarp();
  } else if (warp >= NC) {
    // ------------------------------------------------------------------ producer warps
    // 16-byte cp.async copies, lanes on consecutive chunks of a row (coalesced); keys past
    // the split's end are zero-filled without a read, so masked keys always hold finite
    // values. The NP warps take alternate row groups of a stage (one warp issuing a whole
    // stage's 2048 copies set the first tile's latency); every producer lane's copies of a
    // stage complete on full[slot] (32 NP arrivals).
    constexpr int CPR = D * 2 / 16;          // 16-byte chunks per row (32, 16 or 8)
    constexpr int RPI = 32 / CPR;            // rows per warp instruction (1, 2 or 4)
    static_assert((KTD / RPI) % NP == 0, "whole row groups per producer warp");
    const int pw = warp - NC;                // this warp's row groups: pw, pw + NP, ...
    const int rsub = lane / CPR + pw * RPI, ch = lane % CPR;
    const uint32_t ring_a = smem_u32(ring);
    bool ok = true;
    for (int st = 0; st < nst && ok; ++st) {
      const int slot = st % NSLOT;
      if (st >= NSLOT) ok = mbar_wait(&empty[slot], ((st / NSLOT) - 1) & 1, p.status, kErrWaitKVEmpty);
      if (!ok) break;
      const int kt = k0 + st * KTD;
      uint32_t dk = ring_a + slot * STG + rsub * ROWB + ch * 16;
      const bf16* kp = kb_ptr + int64_t(kt + rsub) * p.k_ss + ch * 8;
      const bf16* vp = vb_ptr + int64_t(kt + rsub) * p.v_ss + ch * 8;
      const int64_t kstep = int64_t(NP * RPI) * p.k_ss, vstep = int64_t(NP * RPI) * p.v_ss;
      int key = kt + rsub;
#pragma unroll 8
      for (int i = 0; i < KTD / RPI / NP; ++i) {
        const bool valid = key < kend;
        cp_async_16_zfill(dk, valid ? kp : kb_ptr, valid);
        cp_async_16_zfill(dk + KTD * ROWB, valid ? vp : vb_ptr, valid);
        dk += NP * RPI * ROWB;
        kp += kstep;
        vp += vstep;
        key += NP * RPI;
      }
      cp_async_mbar_arrive(&full[slot]);
    }
    // never leave with copies in flight: wait (bounded) for this lane's last stages
    for (int st = max(0, nst - NSLOT); st < nst && ok; ++st)
      mbar_wait(&full[st % NSLOT], (st / NSLOT) & 1, p.status, kErrWaitKV);
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ consumer warps
    const int rt = warp % NRT, kslot = (warp / NRT) % KS, ds = warp / (NRT * KS);
    const int gid = lane >> 2, tig = lane & 3;
    const int r0 = rt * 16 + gid, r1 = r0 + 8;             // rows within the group
    const int pr0 = rg * RPG + r0, pr1 = rg * RPG + r1;    // packed rows
    const int nrows = G * qLb;
    const int qi0 = pr0 % qLb, qi1 = pr1 % qLb;
    int kmax0 = Lb - 1, kmax1 = Lb - 1;
    if (p.causal && p.tree_anc == nullptr) {
      kmax0 = Lb - qLb + qi0;
      kmax1 = Lb - qLb + qi1;
    }
    uint32_t anc0 = 0xffffffffu, anc1 = 0xffffffffu;
    if (p.tree_anc != nullptr) {
      anc0 = pr0 < nrows ? p.tree_anc[b * p.qL + qi0] : 0u;
      anc1 = pr1 < nrows ? p.tree_anc[b * p.qL + qi1] : 0u;
    }
    const int tree_lo = Lb - qLb;  // first key governed by the ancestor bits

    // Q fragments in registers
    uint32_t qf[NKK][4];
    {
      const int64_t qb = qbase(p.q_sb, p.q_si);
      const bf16* q0 = pr0 < nrows ? p.q + qb + int64_t(hk * G + pr0 / qLb) * p.q_sh + int64_t(qi0) * p.q_si : nullptr;
      const bf16* q1 = pr1 < nrows ? p.q + qb + int64_t(hk * G + pr1 / qLb) * p.q_sh + int64_t(qi1) * p.q_si : nullptr;
#pragma unroll
      for (int kk = 0; kk < NKK; ++kk) {
        const int d = kk * 16 + 2 * tig;
        qf[kk][0] = q0 ? __ldcg(reinterpret_cast<const unsigned int*>(q0 + d)) : 0u;
        qf[kk][1] = q1 ? __ldcg(reinterpret_cast<const unsigned int*>(q1 + d)) : 0u;
        qf[kk][2] = q0 ? __ldcg(reinterpret_cast<const unsigned int*>(q0 + d + 8)) : 0u;
        qf[kk][3] = q1 ? __ldcg(reinterpret_cast<const unsigned int*>(q1 + d + 8)) : 0u;
      }
    }
    float o[NDT][4];
#pragma unroll
    for (int i = 0; i < NDT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -1e30f, m1 = -1e30f, l0 = 0.f, l1 = 0.f;
    const float sc = p.scale_log2;
    const uint32_t ring_a = smem_u32(ring);

    bool ok = true;  // false once a wait ran out: finish without further waits
    for (int st = 0; st < nst; ++st) {
      const int slot = st % NSLOT;
      if (ok) ok = mbar_wait(&full[slot], (st / NSLOT) & 1, p.status, kErrWaitKV);
      const uint32_t ks_a = ring_a + slot * STG;
      const uint32_t vs_a = ks_a + (TM ? KTD * D * 2 : KTD * ROWB);
      const int kt = k0 + st * KTD;
#pragma unroll
      for (int sub = 0; sub < KPW / KB; ++sub) {
        const int kl = kslot * KPW + sub * KB;   // first key of this step within the tile
        float s[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < NKK; ++kk) {
#pragma unroll
          for (int jp = 0; jp < 2; ++jp) {
            const int mi = lane >> 3;
            const int key = kl + jp * 16 + (mi >> 1) * 8 + (lane & 7);
            const int d = kk * 16 + (mi & 1) * 8;
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4(ks_a + kv_off_in_tile<TM, KTD, ROWB>(key, d), b0, b1, b2, b3);
            mma16816<F16>(s[2 * jp], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
            mma16816<F16>(s[2 * jp + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
          }
        }
        // mask + online softmax (exp2 domain). Steps whose every key is visible to every row of
        // the warp (all but the split's last and the causal / tree boundary) skip the mask.
        float mx0 = -INFINITY, mx1 = -INFINITY;
        const int klast = kt + kl + KB - 1;
        const bool interior = __all_sync(
            0xffffffffu, klast < kend && klast <= min(kmax0, kmax1) &&
                             (p.tree_anc == nullptr || klast < tree_lo));
        if (interior) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            s[j][0] *= sc;
            s[j][1] *= sc;
            s[j][2] *= sc;
            s[j][3] *= sc;
            mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
            mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int key = kt + kl + j * 8 + 2 * tig + (e & 1);
              const bool row1 = e >= 2;
              bool ok = key < kend && key <= (row1 ? kmax1 : kmax0);
              if (p.tree_anc != nullptr && key >= tree_lo)
                ok = ok && (((row1 ? anc1 : anc0) >> (key - tree_lo)) & 1u);
              s[j][e] = ok ? s[j][e] * sc : -INFINITY;
              if (row1) mx1 = fmaxf(mx1, s[j][e]); else mx0 = fmaxf(mx0, s[j][e]);
            }
          }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float f0 = fast_exp2(m0 - mn0), f1 = fast_exp2(m1 - mn1);
        m0 = mn0;
        m1 = mn1;
        float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[j][0] = fast_exp2(s[j][0] - mn0);
          s[j][1] = fast_exp2(s[j][1] - mn0);
          s[j][2] = fast_exp2(s[j][2] - mn1);
          s[j][3] = fast_exp2(s[j][3] - mn1);
          ps0 += s[j][0] + s[j][1];
          ps1 += s[j][2] + s[j][3];
        }
        l0 = l0 * f0 + ps0;
        l1 = l1 * f1 + ps1;
        // once the running maxima settle, every factor is exactly 1: skip the rescale
        if (!__all_sync(0xffffffffu, f0 == 1.f && f1 == 1.f)) {
#pragma unroll
          for (int i = 0; i < NDT; ++i) {
            o[i][0] *= f0; o[i][1] *= f0;
            o[i][2] *= f1; o[i][3] *= f1;
          }
        }
        // O += P . V over two k16 steps of keys
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2) {
          const uint32_t a0 = pack2<F16>(s[2 * k2][0], s[2 * k2][1]);
          const uint32_t a1 = pack2<F16>(s[2 * k2][2], s[2 * k2][3]);
          const uint32_t a2 = pack2<F16>(s[2 * k2 + 1][0], s[2 * k2 + 1][1]);
          const uint32_t a3 = pack2<F16>(s[2 * k2 + 1][2], s[2 * k2 + 1][3]);
          const int mi = lane >> 3;
          const int key = kl + k2 * 16 + (mi & 1) * 8 + (lane & 7);
#pragma unroll
          for (int dt = 0; dt < NDT; dt += 2) {
            const int d = ds * DW + (dt + (mi >> 1)) * 8;
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4_trans(vs_a + kv_off_in_tile<TM, KTD, ROWB>(key, d), b0, b1, b2, b3);
            if (TM && !interior) {
              // keys >= kend hold real cache rows (or the next split's): their P is 0, and
              // their V values are zeroed so that nothing non-finite reaches the MMA. b0 / b2
              // hold keys base + 2 tig, + 1; b1 / b3 hold base + 8 + 2 tig, + 1 (low half first).
              const int kb0 = kt + kl + k2 * 16 + 2 * tig;
              const uint32_t m0 = (kb0 < kend ? 0xFFFFu : 0u) | (kb0 + 1 < kend ? 0xFFFF0000u : 0u);
              const uint32_t m1 = (kb0 + 8 < kend ? 0xFFFFu : 0u) | (kb0 + 9 < kend ? 0xFFFF0000u : 0u);
              b0 &= m0;
              b2 &= m0;
              b1 &= m1;
              b3 &= m1;
            }
            mma16816<F16>(o[dt], a0, a1, a2, a3, b0, b1);
            mma16816<F16>(o[dt + 1], a0, a1, a2, a3, b2, b3);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

    // every warp is past the ring once all consumers reach this barrier
    asm volatile("bar.sync 1, %0;" ::"n"(NC * 32));
    // the key slots k >= 1 hand their partials to the slot-0 warp of the same rows, which
    // merges them in registers (weights once per row, fixed slot order)
    if (kslot > 0) {
      float* myO = bufO + kslot * RPG * D;
#pragma unroll
      for (int dt = 0; dt < NDT; ++dt) {
        const int d = ds * DW + dt * 8 + 2 * tig;
        *reinterpret_cast<float2*>(&myO[r0 * D + d]) = make_float2(o[dt][0], o[dt][1]);
        *reinterpret_cast<float2*>(&myO[r1 * D + d]) = make_float2(o[dt][2], o[dt][3]);
      }
      if (tig == 0 && ds == 0) {
        bufM[kslot * RPG + r0] = m0;
        bufM[kslot * RPG + r1] = m1;
        bufL[kslot * RPG + r0] = l0;
        bufL[kslot * RPG + r1] = l1;
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(NC * 32));
    if (kslot == 0) {
      float M0 = m0, M1 = m1;
#pragma unroll
      for (int k = 1; k < KS; ++k) {
        M0 = fmaxf(M0, bufM[k * RPG + r0]);
        M1 = fmaxf(M1, bufM[k * RPG + r1]);
      }
      float w0[KS], w1[KS];
      w0[0] = fast_exp2(m0 - M0);
      w1[0] = fast_exp2(m1 - M1);
#pragma unroll
      for (int k = 1; k < KS; ++k) {
        w0[k] = fast_exp2(bufM[k * RPG + r0] - M0);
        w1[k] = fast_exp2(bufM[k * RPG + r1] - M1);
      }
#pragma unroll
      for (int dt = 0; dt < NDT; ++dt) {
        const int d = ds * DW + dt * 8 + 2 * tig;
        float a0 = fmaf(w0[0], o[dt][0], 0.f), a1 = fmaf(w0[0], o[dt][1], 0.f);
        float a2 = fmaf(w1[0], o[dt][2], 0.f), a3 = fmaf(w1[0], o[dt][3], 0.f);
#pragma unroll
        for (int k = 1; k < KS; ++k) {
          const float2 u = *reinterpret_cast<const float2*>(&bufO[(k * RPG + r0) * D + d]);
          const float2 v = *reinterpret_cast<const float2*>(&bufO[(k * RPG + r1) * D + d]);
          a0 = fmaf(w0[k], u.x, a0);
          a1 = fmaf(w0[k], u.y, a1);
          a2 = fmaf(w1[k], v.x, a2);
          a3 = fmaf(w1[k], v.y, a3);
        }
        *reinterpret_cast<float2*>(&bufO[r0 * D + d]) = make_float2(a0, a1);
        *reinterpret_cast<float2*>(&bufO[r1 * D + d]) = make_float2(a2, a3);
      }
      if (tig == 0 && ds == 0) {
        float L0 = fmaf(w0[0], l0, 0.f), L1 = fmaf(w1[0], l1, 0.f);
#pragma unroll
        for (int k = 1; k < KS; ++k) {
          L0 = fmaf(w0[k], bufL[k * RPG + r0], L0);
          L1 = fmaf(w1[k], bufL[k * RPG + r1], L1);
        }
        finM[r0] = M0;
        finM[r1] = M1;
        finL[r0] = L0;
        finL[r1] = L1;
      }
    }
  }

  // ------------------------------------------------------------------ split merge + store
  // Every split pushes each of its rows into the CTA of the cluster that owns the row
  // (r % ns): plain stores into distributed shared memory, one cluster barrier, then each
  // owner merges its rows from local shared memory (no round trips on remote loads).
  const int ns = p.ns;
  const int ro = (RPG + ns - 1) / ns;  // rows owned per CTA
  constexpr int RW = D + 4;            // receive row: D accumulators, m, l
  __syncthreads();                     // bufO / finM / finL complete
  if (ns > 1) {
    const uint32_t rbase = smem_u32(recv);
    for (int idx = threadIdx.x; idx < RPG * (D / 4 + 1); idx += blockDim.x) {
      const int r = idx / (D / 4 + 1), c4 = idx - r * (D / 4 + 1);
      const int owner = r % ns, rl = r / ns;
      const uint32_t dst = mapa_shared(rbase + uint32_t(((sidx_c * ro + rl) * RW + c4 * 4) * 4), owner);
      if (c4 < D / 4)
        st_dsmem_f4(dst, *reinterpret_cast<const float4*>(&bufO[r * D + c4 * 4]));
      else
        st_dsmem_f4(dst, make_float4(finM[r], finL[r], 0.f, 0.f));
    }
    cluster_sync_all();  // pushes visible to their owners
  }
  const int64_t ob = qbase(p.o_sb, p.o_si);
  const int nrows = G * qLb;
  for (int idx = threadIdx.x; idx < ro * (D / 4); idx += blockDim.x) {
    const int rl = idx / (D / 4), d4 = (idx % (D / 4)) * 4;
    const int r = ns > 1 ? sidx_c + rl * ns : rl;
    if (r >= RPG) continue;
    const int prow = rg * RPG + r;
    if (prow >= nrows) continue;
    float M = -1e30f, Lsum = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ns > 1) {
      for (int c = 0; c < ns; ++c) M = fmaxf(M, recv[(c * ro + rl) * RW + D]);
      for (int c = 0; c < ns; ++c) {
        const float* src = recv + (c * ro + rl) * RW;
        const float w = fast_exp2(src[D] - M);
        Lsum += w * src[D + 1];
        const float4 v = *reinterpret_cast<const float4*>(&src[d4]);
        acc.x += w * v.x; acc.y += w * v.y; acc.z += w * v.z; acc.w += w * v.w;
      }
    } else {
      M = finM[r];
      Lsum = finL[r];
      acc = *reinterpret_cast<const float4*>(&bufO[r * D + d4]);
    }
    if (p.ng > 1) {
      // unnormalized partial for the cross-cluster merge
      float* w = p.ws + ((int64_t(bhr) * p.ng + g_grp) * RPG + r) * kWsRow<D>;
      *reinterpret_cast<float4*>(&w[d4]) = acc;
      if (d4 == 0) {
        w[D] = M;
        w[D + 1] = Lsum;
      }
    } else {
      const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
      const int h = hk * G + prow / qLb, i = prow % qLb;
      bf16* dst = p.o + ob + int64_t(h) * p.o_sh + int64_t(i) * p.o_si + d4;
      uint2 pk;
      pk.x = pack2<F16>(acc.x * inv, acc.y * inv);
      pk.y = pack2<F16>(acc.z * inv, acc.w * inv);
      *reinterpret_cast<uint2*>(dst) = pk;
    }
  }
}

template <int D, int NRT, int KS, int DS, bool F16, int QB = 0>
__global__ void __launch_bounds__((NRT * KS * DS + n_producers<QB>()) * 32)
    attn_kernel(const __grid_constant__ AttnParams p) {
  attn_body<D, NRT, KS, DS, F16, QB, false>(nullptr, nullptr, p);
}

template <int D, int NRT, int KS, int DS, bool F16>
__global__ void __launch_bounds__((NRT * KS * DS + 1) * 32)
    attn_kernel_tma(const __grid_constant__ CUtensorMap kmap,
                    const __grid_constant__ CUtensorMap vmap, const __grid_constant__ AttnParams p) {
  attn_body<D, NRT, KS, DS, F16, 0, true>(&kmap, &vmap, p);
}

// Cross-cluster merge of the ng partials (only when ng > 1): one warp per packed row, every
// lane loads all ng partials of its D/32 columns at once (no dependent load chains).
constexpr int kMergeRows = 8;  // rows (warps) per block

template <int D, bool F16>
__global__ void __launch_bounds__(kMergeRows * 32) attn_merge_kernel(const AttnParams p, int rpg) {
  pdl_launch_dependents();
  pdl_wait();
  constexpr int DPL = D / 32;  // columns per lane (8, 4 or 2)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grow = blockIdx.x * kMergeRows + warp;  // (bhr, r) flattened
  const int bhr = grow / rpg, r = grow - bhr * rpg;
  if (bhr >= p.B * p.Hk * p.nrg) return;
  const int rg = bhr % p.nrg, bh = bhr / p.nrg;
  const int hk = bh % p.Hk, b = bh / p.Hk;
  const int G = p.Hq / p.Hk;
  const int qLb = p.q_len ? p.q_len[b] : p.qL;
  const int prow = rg * rpg + r;
  if (prow >= G * qLb) return;
  const float* base = p.ws + (int64_t(bhr) * p.ng * rpg + r) * kWsRow<D>;
  const int64_t gstride = int64_t(rpg) * kWsRow<D>;
  // the partials' maxima: lane g holds group g's (m, l)
  float mg = -1e30f, lg = 0.f;
  if (lane < p.ng) {
    const float2 ml = *reinterpret_cast<const float2*>(base + lane * gstride + D);
    mg = ml.x;
    lg = ml.y;
  }
  float M = mg;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  const float wl = lane < p.ng ? fast_exp2(mg - M) : 0.f;
  float L = wl * lg;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  float acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
  for (int g = 0; g < p.ng; ++g) {
    const float w = __shfl_sync(0xffffffffu, wl, g);
    const float* src = base + g * gstride + lane * DPL;
#pragma unroll
    for (int c = 0; c < DPL; c += 2) {
      const float2 v = *reinterpret_cast<const float2*>(src + c);
      acc[c] += w * v.x;
      acc[c + 1] += w * v.y;
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  const int h = hk * G + prow / qLb, i = prow % qLb;
  bf16* dst = p.o + q_base(p, b, p.o_sb, p.o_si) + int64_t(h) * p.o_sh + int64_t(i) * p.o_si + lane * DPL;
#pragma unroll
  for (int c = 0; c < DPL; c += 2)
    *reinterpret_cast<uint32_t*>(dst + c) = pack2<F16>(acc[c] * inv, acc[c + 1] * inv);
}

// ------------------------------------------------------------------------------ host side

// warps sharing a row tile's columns: 2 for head_dim 256 (each keeps half of the output)
__host__ __device__ constexpr int dsplit(int d) { return d > 128 ? 2 : 1; }

// Clusters of `cs` CTAs of the attention kernel for (D, nrt, ks) that the device runs at once.
template <int D, int NRT, int KS>
static int max_clusters_t(int cs) {
  constexpr int DS = dsplit(D);
  auto kern = attn_kernel<D, NRT, KS, DS, false>;  // same shape for both input types
  constexpr int smem = attn_smem_bytes<D, NRT, KS>();
  // a refused query: portable sizes fall back to one CTA per SM, larger ones are not used
  const int fallback = cs <= 8 ? sm_count(current_device()) / cs : 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
      cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
    cudaGetLastError();
    return fallback;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cs, 1, 1);
  cfg.blockDim = dim3((NRT * KS * DS + n_producers<0>()) * 32);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = cs;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int c = 0;
  if (cudaOccupancyMaxActiveClusters(&c, kern, &cfg) != cudaSuccess || c <= 0) {
    cudaGetLastError();
    c = fallback;
  }
  return c;
}

static int max_clusters(int D, int nrt, int ks, int cs) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int>, int> cache;
  const auto key = std::make_tuple(current_device(), D, nrt, ks, cs);
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int n;
  if (D == 64) {
    n = nrt == 1 ? max_clusters_t<64, 1, 2>(cs) : nrt == 2 ? max_clusters_t<64, 2, 2>(cs)
        : nrt == 4 ? max_clusters_t<64, 4, 2>(cs) : max_clusters_t<64, 8, 1>(cs);
  } else if (D == 128) {
    n = nrt == 1 ? max_clusters_t<128, 1, 2>(cs) : nrt == 2 ? max_clusters_t<128, 2, 2>(cs)
        : nrt == 4 ? max_clusters_t<128, 4, 2>(cs) : max_clusters_t<128, 8, 1>(cs);
  } else {
    n = nrt == 1 ? max_clusters_t<256, 1, 1>(cs) : nrt == 2 ? max_clusters_t<256, 2, 1>(cs)
        : max_clusters_t<256, 4, 1>(cs);
  }
  std::lock_guard<std::mutex> g(mu);
  cache[key] = n;
  return n;
}

AttnPlan plan(int B, int Hq, int Hk, int qL, int D, int L) {
  AttnPlan pl;
  const int rows = (Hq / Hk) * qL;
  const int tiles = (rows + 15) / 16;
  int nrt;
  if (tiles <= 1) nrt = 1;
  else if (tiles <= 2) nrt = 2;
  else if (tiles <= 4) nrt = 4;
  else nrt = 8;
  // head_dim 256: at most 4 row tiles per CTA (shared memory) and one key slot (32-key stages)
  if (D > 128) nrt = std::min(nrt, 4);
  // Up to 4k keys, two row tiles per CTA (twice the row groups, each streaming the head's keys,
  // the second from L2) beat four. Measured at 16 rows x 4 heads per KV head, 1k / 2k / 4k keys:
  // 10.4 / 12.9 / 18.4 us with four row tiles, 8.9 / 11.9 / 16.9 us with two; at 32k keys four
  // win (56.8 against 66.5 us). DSPARK_ATTN_NRT (1, 2 or 4) forces a cap, for tuning.
  const int force_nrt = env_int("DSPARK_ATTN_NRT", 0);
  if (force_nrt == 1 || force_nrt == 2 || (force_nrt == 4 && D <= 128))
    nrt = std::min(nrt, force_nrt);
  else if (D <= 128 && L <= 4096)
    nrt = std::min(nrt, 2);
  pl.nrt = nrt;
  pl.ks = (nrt >= 8 || D > 128) ? 1 : 2;
  const int kt = ktile(D);
  pl.nrg = (tiles + nrt - 1) / nrt;
  const int heads = B * Hk * pl.nrg;
  // key splits per head: as many CTAs as run at once in a single wave (clusters of ns CTAs
  // merge their splits through distributed shared memory; ns <= 16, 16 being a non-portable
  // size the device may refuse, chosen by how many such clusters the device co-schedules),
  // each streaming >= 128 keys; cluster groups merge through the workspace. At equal split
  // counts the larger cluster wins: fewer groups, and with one group no merge kernel at all.
  const int max_splits = std::max(1, L / 128);
  const int force = env_int("DSPARK_ATTN_SPLITS", 0);
  int ns = 1, ng = 1;
  if (force > 0) {
    ns = std::min(force, 8);
    ng = (force + ns - 1) / ns;
  } else {
    // Modelled as: every CTA streams ceil(L / splits / 64) key tiles at ~1.3 us each (64 packed
    // rows, measured on B200), and a second cluster group adds the workspace merge pass
    // (~7 us: the merge launch and its round trip); the fixed per-launch costs are common to
    // every plan. Cluster groups are limited to what the device co-schedules in one wave.
    const double t_tile = 1.3, t_merge = 7.0;
    double best = 1e30;
    for (int c : {16, 8, 6, 4, 3, 2, 1}) {
      if (c > max_splits) continue;
      const int fit = c == 1 ? sm_count(current_device()) / std::max(1, heads)
                             : max_clusters(D, nrt, pl.ks, c) / std::max(1, heads);
      const int gmax = std::min({fit, max_splits / c, 32});
      for (int g = 1; g <= gmax; ++g) {
        const int keys = (L + c * g - 1) / (c * g);
        const int tiles = (keys + KT - 1) / KT;  // 64-key units of work
        const double t = tiles * t_tile + (g > 1 ? t_merge : 0.0);
        if (t < best - 1e-9) {  // ties keep the larger cluster (tried first)
          best = t;
          ns = c;
          ng = g;
        }
      }
    }
  }
  int chunk = ((L + ns * ng - 1) / (ns * ng) + kt - 1) / kt * kt;
  chunk = std::max(chunk, kt);
  // drop splits that would start past the end
  while (ns * ng > 1 && (ns * ng - 1) * chunk >= L) {
    if (ng > 1) --ng; else --ns;
  }
  pl.ns = std::max(1, ns);
  pl.ng = std::max(1, std::min(ng, 32));  // the merge kernel holds one group per lane
  pl.chunk = ((L + pl.ns * pl.ng - 1) / (pl.ns * pl.ng) + kt - 1) / kt * kt;
  pl.chunk = std::max(pl.chunk, kt);
  return pl;
}

size_t workspace_bytes(const AttnPlan& pl, int B, int Hk, int D) {
  if (pl.ng <= 1) return 0;
  return size_t(B) * Hk * pl.nrg * pl.ng * (pl.nrt * 16) * (D + 4) * sizeof(float);
}

// Tensor maps over K and V as [B][Hk][L][D] (dims innermost first), boxes of [KTD keys x 64
// dims] with the 128-byte swizzle. Only for the dense bf16 / fp16 layout (no per-request cache
// offsets) and when the driver accepts the strides; otherwise the cp.async producer serves.
template <int D>
static bool kv_maps(const AttnParams& p, CUtensorMap* km, CUtensorMap* vm) {
  if (p.qbits || p.kv_off || env_int("DSPARK_ATTN_TMA", 0) == 0) return false;
  const uint64_t bs_k = uint64_t(p.B > 1 ? p.k_sb : p.k_sh * p.Hk) * 2;
  const uint64_t bs_v = uint64_t(p.B > 1 ? p.v_sb : p.v_sh * p.Hk) * 2;
  const uint64_t dims[4] = {uint64_t(D), uint64_t(p.L), uint64_t(p.Hk), uint64_t(p.B)};
  const uint64_t ks[3] = {uint64_t(p.k_ss) * 2, uint64_t(p.k_sh) * 2, bs_k};
  const uint64_t vs[3] = {uint64_t(p.v_ss) * 2, uint64_t(p.v_sh) * 2, bs_v};
  const uint32_t box[4] = {64u, uint32_t(ktile(D)), 1u, 1u};
  return encode_tmap_nd(km, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, p.k, dims, ks, box,
                        CU_TENSOR_MAP_SWIZZLE_128B) &&
         encode_tmap_nd(vm, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, p.v, dims, vs, box,
                        CU_TENSOR_MAP_SWIZZLE_128B);
}

template <typename Kern>
static cudaError_t configure_attn(Kern kern, int smem) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
}

template <int D, int NRT, int KS, bool F16, int QB = 0>
static int launch_attn(const AttnParams& p, const AttnPlan& pl, cudaStream_t s) {
  constexpr int DS = dsplit(D);
  constexpr int smem = attn_smem_bytes<D, NRT, KS>();
  dim3 grid(pl.ns, p.B * p.Hk * pl.nrg, pl.ng);
  dim3 block((NRT * KS * DS + n_producers<QB>()) * 32);
  const dim3 block_tma((NRT * KS * DS + 1) * 32);  // one TMA producer warp
  CUtensorMap km, vm;
  bool tma = false;
  if constexpr (QB == 0) tma = kv_maps<D>(p, &km, &vm);
  if (tma) {
    if constexpr (QB == 0) {
      auto kern = attn_kernel_tma<D, NRT, KS, DS, F16>;
      DSPARK_CUDA_TRY(configure_once(reinterpret_cast<const void*>(kern), 1,
                                     [&] { return configure_attn(kern, smem); }),
                      "attn: set smem / cluster attributes");
      DSPARK_CUDA_TRY(launch_ex(kern, grid, block_tma, smem, s, pl.ns, true, km, vm, p), "attn: launch");
    }
  } else {
    auto kern = attn_kernel<D, NRT, KS, DS, F16, QB>;
    DSPARK_CUDA_TRY(configure_once(reinterpret_cast<const void*>(kern), 1,
                                   [&] { return configure_attn(kern, smem); }),
                    "attn: set smem / cluster attributes");
    DSPARK_CUDA_TRY(launch_ex(kern, grid, block, smem, s, pl.ns, true, p), "attn: launch");
  }
  if (pl.ng > 1) {
    const int rows = p.B * p.Hk * pl.nrg * NRT * 16;
    DSPARK_CUDA_TRY(launch_ex(attn_merge_kernel<D, F16>,
                              dim3((rows + kMergeRows - 1) / kMergeRows), dim3(kMergeRows * 32),
                              0, s, 1, true, p, NRT * 16),
                    "attn: merge launch");
  }
  return DSPARK_OK;
}

template <int D, bool F16>
static int dispatch_d(const AttnParams& p, const AttnPlan& pl, cudaStream_t s) {
  if constexpr (D > 128) {
    if (pl.nrt == 1 && pl.ks == 1) return launch_attn<D, 1, 1, F16>(p, pl, s);
    if (pl.nrt == 2 && pl.ks == 1) return launch_attn<D, 2, 1, F16>(p, pl, s);
    if (pl.nrt == 4 && pl.ks == 1) return launch_attn<D, 4, 1, F16>(p, pl, s);
  } else {
    if (pl.nrt == 1 && pl.ks == 2) return launch_attn<D, 1, 2, F16>(p, pl, s);
    if (pl.nrt == 2 && pl.ks == 2) return launch_attn<D, 2, 2, F16>(p, pl, s);
    if (pl.nrt == 4 && pl.ks == 2) return launch_attn<D, 4, 2, F16>(p, pl, s);
    if (pl.nrt == 8 && pl.ks == 1) return launch_attn<D, 8, 1, F16>(p, pl, s);
  }
  return fail(DSPARK_ERR_UNSUPPORTED, "attn: no kernel for head_dim %d, %d row tiles x %d key slots",
              D, pl.nrt, pl.ks);
}

template <int D, int QB>
static int dispatch_q(const AttnParams& p, const AttnPlan& pl, cudaStream_t s) {
  if (pl.nrt == 1 && pl.ks == 2) return launch_attn<D, 1, 2, false, QB>(p, pl, s);
  if (pl.nrt == 2 && pl.ks == 2) return launch_attn<D, 2, 2, false, QB>(p, pl, s);
  if (pl.nrt == 4 && pl.ks == 2) return launch_attn<D, 4, 2, false, QB>(p, pl, s);
  if (pl.nrt == 8 && pl.ks == 1) return launch_attn<D, 8, 1, false, QB>(p, pl, s);
  return fail(DSPARK_ERR_UNSUPPORTED, "attn: no quantized-KV kernel for %d row tiles", pl.nrt);
}

template <bool F16>
static int dispatch_t(const AttnParams& p, const AttnPlan& pl, cudaStream_t s) {
  if (p.D == 64) return dispatch_d<64, F16>(p, pl, s);
  if (p.D == 128) return dispatch_d<128, F16>(p, pl, s);
  return dispatch_d<256, F16>(p, pl, s);
}

int run(AttnParams p, const AttnPlan* plan_in, cudaStream_t stream) {
  if (p.B <= 0 || p.Hq <= 0 || p.Hk <= 0 || p.Hq % p.Hk || p.qL <= 0 || p.L <= 0)
    return fail(DSPARK_ERR_ARG, "attn: bad shape B=%d Hq=%d Hk=%d qL=%d L=%d", p.B, p.Hq, p.Hk, p.qL, p.L);
  if (p.D != 64 && p.D != 128 && p.D != 256)
    return fail(DSPARK_ERR_UNSUPPORTED, "attn: head_dim %d not supported (64, 128, 256)", p.D);
  if (p.qL > 32 && p.tree_anc)
    return fail(DSPARK_ERR_UNSUPPORTED, "attn: tree verify supports at most 32 rows");
  if (p.qbits) {
    if (p.qbits != 4 && p.qbits != 8) return fail(DSPARK_ERR_UNSUPPORTED, "attn: %d-bit KV", p.qbits);
    if (p.D != 64 && p.D != 128)
      return fail(DSPARK_ERR_UNSUPPORTED, "attn: quantized KV needs head_dim 64 or 128 (got %d)", p.D);
    if (p.f16 || p.kv_off || p.tree_anc)
      return fail(DSPARK_ERR_UNSUPPORTED, "attn: quantized KV serves bf16, dense rows, causal / full rules");
    if (!p.kq || !p.vq || !p.ksc || !p.kbi || !p.vsc || !p.vbi)
      return fail(DSPARK_ERR_ARG, "attn: null quantized K/V pointer");
    const uintptr_t qa = reinterpret_cast<uintptr_t>(p.kq) | reinterpret_cast<uintptr_t>(p.vq);
    if ((qa & 15) || ((p.kq_sb | p.kq_sh | p.kq_ss) & 3))
      return fail(DSPARK_ERR_UNSUPPORTED, "attn: K/V code rows must be 16-byte aligned");
  } else {
    const uintptr_t al = reinterpret_cast<uintptr_t>(p.k) | reinterpret_cast<uintptr_t>(p.v);
    if ((al & 15) || ((p.k_sb | p.k_sh | p.k_ss | p.v_sb | p.v_sh | p.v_ss) & 7))
      return fail(DSPARK_ERR_UNSUPPORTED, "attn: K/V rows must be 16-byte aligned (strides %% 8 == 0)");
  }
  if ((reinterpret_cast<uintptr_t>(p.q) & 3) || (reinterpret_cast<uintptr_t>(p.o) & 7) ||
      ((p.q_sb | p.q_sh | p.q_si) & 1) || ((p.o_sb | p.o_sh | p.o_si) & 3))
    return fail(DSPARK_ERR_UNSUPPORTED, "attn: q rows need 4-byte and output rows 8-byte alignment");
  if (!p.kv_len && p.causal && !p.tree_anc && p.qL > p.L)
    return fail(DSPARK_ERR_ARG, "attn: causal verify needs qL <= L (qL=%d L=%d)", p.qL, p.L);
  AttnPlan pl = plan_in ? *plan_in : plan(p.B, p.Hq, p.Hk, p.qL, p.D, p.L);
  p.nrg = pl.nrg;
  p.ns = pl.ns;
  p.ng = pl.ng;
  p.chunk = pl.chunk;
  if (pl.ng > 32) return fail(DSPARK_ERR_UNSUPPORTED, "attn: at most 32 cluster groups (got %d)", pl.ng);
  if (pl.ns < 1 || pl.ns > 16)
    return fail(DSPARK_ERR_UNSUPPORTED, "attn: cluster of %d key splits (1..16)", pl.ns);
  if (pl.ng > 1 && p.ws == nullptr)
    return fail(DSPARK_ERR_ARG, "attn: this launch needs a workspace of %zu bytes",
                workspace_bytes(pl, p.B, p.Hk, p.D));
  if (p.status == nullptr) p.status = status_word(current_device());
  if (p.qbits) {
    if (p.D == 64) return p.qbits == 8 ? dispatch_q<64, 8>(p, pl, stream) : dispatch_q<64, 4>(p, pl, stream);
    return p.qbits == 8 ? dispatch_q<128, 8>(p, pl, stream) : dispatch_q<128, 4>(p, pl, stream);
  }
  return p.f16 ? dispatch_t<true>(p, pl, stream) : dispatch_t<false>(p, pl, stream);
}

}  // namespace attn
}  // namespace dspark
