// K3 / K4 and forward glue: KV append / rollback / row move, argmax + greedy accept,
// ragged request packing, quantized embedding, RMSNorm.
//
// These are the integer / byte paths around the verify forward (HBM- or latency-bound):
// coalesced 16-byte accesses, one CTA per independent unit, no scratch memory.
#include "common.cuh"
#include "host_common.h"
#include "ops.h"

namespace dspark {
namespace ops {

// ------------------------------------------------------------------------ KV append

// grid (T, H, B); block: row_bytes/16 threads, each moving 16 bytes. Strides in bytes.
__global__ void kv_append_kernel(const uint8_t* kn, int64_t kn_b, int64_t kn_h, int64_t kn_t,
                                 const uint8_t* vn, int64_t vn_b, int64_t vn_h, int64_t vn_t,
                                 uint8_t* kc, int64_t kc_b, int64_t kc_h, int64_t kc_t, uint8_t* vc,
                                 int64_t vc_b, int64_t vc_h, int64_t vc_t, const int32_t* lens,
                                 int row_bytes, int cap, int* status) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int pos = lens[b] + t;
  if (pos >= cap || pos < 0) {
    if (threadIdx.x == 0) report_error(status, 0x201);
    return;
  }
  const int d = threadIdx.x * 16;
  if (d >= row_bytes) return;
  const uint4 kv = *reinterpret_cast<const uint4*>(kn + b * kn_b + h * kn_h + t * kn_t + d);
  const uint4 vv = *reinterpret_cast<const uint4*>(vn + b * vn_b + h * vn_h + t * vn_t + d);
  *reinterpret_cast<uint4*>(kc + b * kc_b + h * kc_h + int64_t(pos) * kc_t + d) = kv;
  *reinterpret_cast<uint4*>(vc + b * vc_b + h * vc_h + int64_t(pos) * vc_t + d) = vv;
}

// lens[b] += T after the append (separate launch: the append kernel reads lens)
__global__ void lens_add_kernel(int32_t* lens, int B, int T, int cap) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) lens[b] = min(cap, lens[b] + T);
}

__global__ void kv_rollback_kernel(int32_t* lens, const int32_t* n_rej, int B) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) lens[b] = max(0, lens[b] - n_rej[b]);
}

// grid (chunks of rows, H); copies row src's live positions onto row dst. Strides in bytes.
__global__ void kv_move_kernel(uint8_t* kc, int64_t kc_b, int64_t kc_h, int64_t kc_t, uint8_t* vc,
                               int64_t vc_b, int64_t vc_h, int64_t vc_t, int32_t* lens, int src,
                               int dst, int row_bytes) {
  pdl_launch_dependents();
  pdl_wait();
  const int n = lens[src];
  const int h = blockIdx.y;
  const int per_row = row_bytes / 16;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n * per_row; i += gridDim.x * blockDim.x) {
    const int pos = i / per_row, d = (i % per_row) * 16;
    const int64_t so = int64_t(src) * kc_b + h * kc_h + int64_t(pos) * kc_t + d;
    const int64_t dofs = int64_t(dst) * kc_b + h * kc_h + int64_t(pos) * kc_t + d;
    *reinterpret_cast<uint4*>(kc + dofs) = *reinterpret_cast<const uint4*>(kc + so);
    const int64_t vso = int64_t(src) * vc_b + h * vc_h + int64_t(pos) * vc_t + d;
    const int64_t vdo = int64_t(dst) * vc_b + h * vc_h + int64_t(pos) * vc_t + d;
    *reinterpret_cast<uint4*>(vc + vdo) = *reinterpret_cast<const uint4*>(vc + vso);
  }
}

__global__ void kv_move_lens_kernel(int32_t* lens, int src, int dst) {
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x == 0 && src != dst) {
    lens[dst] = lens[src];
    lens[src] = 0;
  }
}

// ------------------------------------------------------------------------ argmax / accept

__device__ __forceinline__ void better(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

// one CTA per row; first index wins ties (numpy / mx.argmax convention)
__global__ void __launch_bounds__(1024) argmax_kernel(const bf16* logits, int64_t ld, int V,
                                                      int32_t* tt) {
  pdl_launch_dependents();
  pdl_wait();
  const bf16* row = logits + int64_t(blockIdx.x) * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  const int nv = V / 8;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const uint4 q = __ldcg(reinterpret_cast<const uint4*>(row + i * 8));
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      better(bv, bi, bf16_lo(w[e]), i * 8 + 2 * e);
      better(bv, bi, bf16_hi(w[e]), i * 8 + 2 * e + 1);
    }
  }
  for (int i = nv * 8 + threadIdx.x; i < V; i += blockDim.x) better(bv, bi, bf2f(row[i]), i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, ov, oi);
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    bv = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      better(bv, bi, ov, oi);
    }
    if (lane == 0) tt[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
  }
}

__global__ void accept_kernel(const int32_t* tt, const int32_t* ids, const int32_t* cu, int B,
                              int32_t* n_accept, int32_t* next_tok, int32_t* lens) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int r0 = cu[b], r1 = cu[b + 1];
  if (r1 <= r0) {  // an idle slot (no rows this step): nothing accepted, length unchanged
    if (n_accept) n_accept[b] = 0;
    if (next_tok) next_tok[b] = -1;
    return;
  }
  const int cap = r1 - r0 - 1;
  int n = 0;
  while (n < cap && ids[r0 + 1 + n] == tt[r0 + n]) ++n;
  if (n_accept) n_accept[b] = n;
  if (next_tok) next_tok[b] = tt[r0 + n];
  if (lens) lens[b] = max(0, lens[b] - (cap - n));
}

// ------------------------------------------------------------------------ ragged packing

// single CTA: prefix sum of block lengths, then one thread per packed row
__global__ void __launch_bounds__(1024) pack_kernel(const int32_t* block_len, const int32_t* kv_len,
                                                    const int64_t* slot_off, const int32_t* ids_pad,
                                                    int t_max, int B, int r_max, int32_t* cu,
                                                    int32_t* row_pos, int64_t* row_kv,
                                                    int32_t* row_req, int32_t* ids,
                                                    int32_t* kv_len_new) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ int32_t s_cu[4097];
  __shared__ int32_t warp_tot[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // blocked scan: each thread owns a contiguous run of requests
  const int per = (B + blockDim.x - 1) / blockDim.x;
  const int b0 = min(B, tid * per), b1 = min(B, b0 + per);
  int local = 0;
  for (int b = b0; b < b1; ++b) local += block_len[b];
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int w = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) warp_tot[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  int run = incl - local + (warp > 0 ? warp_tot[warp - 1] : 0);
  for (int b = b0; b < b1; ++b) {
    s_cu[b] = run;
    run += block_len[b];
  }
  if (tid == blockDim.x - 1 || (b1 == B && b0 < b1)) s_cu[B] = run;
  if (B == 0 && tid == 0) s_cu[0] = 0;
  __syncthreads();
  for (int b = tid; b <= B; b += blockDim.x) cu[b] = s_cu[b];
  for (int b = tid; b < B; b += blockDim.x) kv_len_new[b] = kv_len[b] + block_len[b];
  const int R = s_cu[B];
  for (int r = tid; r < r_max; r += blockDim.x) {
    if (r < R) {
      // request owning row r: largest b with s_cu[b] <= r
      int lo = 0, hi = B - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_cu[mid] <= r) lo = mid; else hi = mid - 1;
      }
      const int i = r - s_cu[lo];
      row_req[r] = lo;
      row_pos[r] = kv_len[lo] + i;
      row_kv[r] = slot_off[lo];
      ids[r] = i < t_max ? ids_pad[int64_t(lo) * t_max + i] : 0;
    } else {
      row_req[r] = 0;
      row_pos[r] = B > 0 ? kv_len[0] : 0;
      row_kv[r] = B > 0 ? slot_off[0] : 0;
      ids[r] = 0;
    }
  }
}

__global__ void batch_mask_kernel(const int32_t* off, int B, int T, int Lcur, uint8_t* mask) {
  const int64_t total = int64_t(B) * T * Lcur;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int j = int(i % Lcur);
    const int t = int((i / Lcur) % T);
    const int b = int(i / (int64_t(Lcur) * T));
    mask[i] = j <= off[b] + t ? 1 : 0;
  }
}

// ------------------------------------------------------------------------ embed / rmsnorm

// grid M; block 256. h[m] = dequant(table[ids[m]]); ssq[m] = sum(h^2)
template <int BITS>
__global__ void embed_kernel(const int32_t* ids, const uint32_t* wq, const bf16* sc, const bf16* bi,
                             int H, int V, bf16* h, float* ssq) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  const int64_t row = min(max(ids[m], 0), V - 1);  // out-of-vocabulary ids read row 0 / V-1
  const int wpr = H * BITS / 32;
  const int G = H / 64;
  float ss = 0.f;
  constexpr int PER = 32 / BITS;  // values per word
  for (int w = threadIdx.x; w < wpr; w += blockDim.x) {
    const uint32_t q = wq[row * wpr + w];
    const int k0 = w * PER;
    const int g = k0 / 64;
    const float s = bf2f(sc[row * G + g]), b = bf2f(bi[row * G + g]);
    float v[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      v[e] = round_bf16(fmaf(s, float((q >> (BITS * e)) & ((1u << BITS) - 1u)), b));
      ss += v[e] * v[e];
    }
#pragma unroll
    for (int e = 0; e < PER; e += 2)
      *reinterpret_cast<uint32_t*>(h + int64_t(m) * H + k0 + e) = pack_bf16x2(v[e], v[e + 1]);
  }
  if (ssq == nullptr) return;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += part[i];
    ssq[m] = t;
  }
}

// grid M; block 256
__global__ void rmsnorm_kernel(const bf16* x, int64_t ldx, int H, const bf16* w, float eps,
                               bf16* out, int64_t ldo) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  const bf16* xr = x + int64_t(m) * ldx;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = bf2f(xr[i]);
    ss += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float part[32];
  __shared__ float rs;
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += part[i];
    rs = rsqrtf(t / float(H) + eps);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    out[int64_t(m) * ldo + i] = __float2bfloat16_rn(bf2f(xr[i]) * rs * bf2f(w[i]));
}

// single-request packing for the verify forward
__global__ void verify_prepare_kernel(int32_t* len, int R, int32_t* row_pos, int64_t* row_kv,
                                      int32_t* kv_len, int32_t* row_start, int32_t* q_len,
                                      int64_t* kv_off) {
  pdl_launch_dependents();
  pdl_wait();
  const int L0 = len[0];
  __syncthreads();  // every thread has read L0 before it is advanced
  const int m = threadIdx.x;
  if (m < R) {
    row_pos[m] = L0 + m;
    row_kv[m] = 0;
  }
  if (m == 0) {
    kv_len[0] = L0 + R;
    len[0] = L0 + R;  // the forward appends the block's K/V
    row_start[0] = 0;
    q_len[0] = R;
    kv_off[0] = 0;
  }
}

__global__ void inv_freq_kernel(float* inv_freq, int half, float log2_theta) {
  const int i = threadIdx.x;
  if (i < half) inv_freq[i] = exp2f(-float(i) / float(half) * log2_theta);
}

// ------------------------------------------------------------------------ host wrappers

int kv_append(const KvAppend& a, cudaStream_t s) {
  const int rb = a.D * a.esize;
  if (rb % 16 || rb > 16 * 1024)
    return fail(DSPARK_ERR_UNSUPPORTED, "kv_append: row of %d bytes (needs a multiple of 16)", rb);
  if (a.B <= 0 || a.H <= 0 || a.T <= 0) return fail(DSPARK_ERR_ARG, "kv_append: empty shape");
  const uintptr_t al = reinterpret_cast<uintptr_t>(a.kn) | reinterpret_cast<uintptr_t>(a.vn) |
                       reinterpret_cast<uintptr_t>(a.kc) | reinterpret_cast<uintptr_t>(a.vc);
  int64_t st_or = 0;
  for (int i = 0; i < 3; ++i) st_or |= a.kn_s[i] | a.vn_s[i] | a.kc_s[i] | a.vc_s[i];
  if ((al & 15) || ((st_or * a.esize) & 15))
    return fail(DSPARK_ERR_UNSUPPORTED, "kv_append: rows must be 16-byte aligned");
  int* st = status_word(current_device());
  const int64_t e = a.esize;
  DSPARK_CUDA_TRY(launch_ex(kv_append_kernel, dim3(a.T, a.H, a.B), dim3(rb / 16), 0, s, 1, true,
                            (const uint8_t*)a.kn, a.kn_s[0] * e, a.kn_s[1] * e, a.kn_s[2] * e,
                            (const uint8_t*)a.vn, a.vn_s[0] * e, a.vn_s[1] * e, a.vn_s[2] * e,
                            (uint8_t*)a.kc, a.kc_s[0] * e, a.kc_s[1] * e, a.kc_s[2] * e,
                            (uint8_t*)a.vc, a.vc_s[0] * e, a.vc_s[1] * e, a.vc_s[2] * e,
                            (const int32_t*)a.lens, rb, a.cap, st),
                  "kv_append");
  DSPARK_CUDA_TRY(launch_ex(lens_add_kernel, dim3((a.B + 255) / 256), dim3(256), 0, s, 1, true,
                            a.lens, a.B, a.T, a.cap),
                  "kv_append lens");
  return DSPARK_OK;
}

int kv_rollback(int32_t* lens, const int32_t* n_rej, int B, cudaStream_t s) {
  if (B <= 0) return DSPARK_OK;
  DSPARK_CUDA_TRY(launch_ex(kv_rollback_kernel, dim3((B + 255) / 256), dim3(256), 0, s, 1, true,
                            lens, n_rej, B),
                  "kv_rollback");
  return DSPARK_OK;
}

int kv_move_row(void* kc, const int64_t* kc_s, void* vc, const int64_t* vc_s, int32_t* lens,
                int src, int dst, int H, int D, int esize, int max_len, cudaStream_t s) {
  const int rb = D * esize;
  if (rb % 16) return fail(DSPARK_ERR_UNSUPPORTED, "kv_move_row: row of %d bytes", rb);
  const uintptr_t al = reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc);
  if ((al & 15) || (((kc_s[0] | kc_s[1] | kc_s[2] | vc_s[0] | vc_s[1] | vc_s[2]) * esize) & 15))
    return fail(DSPARK_ERR_UNSUPPORTED, "kv_move_row: rows must be 16-byte aligned");
  if (src == dst) return DSPARK_OK;
  const int64_t e = esize;
  const int blocks = std::max(1, std::min(1024, (max_len * (rb / 16) + 255) / 256));
  DSPARK_CUDA_TRY(launch_ex(kv_move_kernel, dim3(blocks, H), dim3(256), 0, s, 1, true,
                            (uint8_t*)kc, kc_s[0] * e, kc_s[1] * e, kc_s[2] * e, (uint8_t*)vc,
                            vc_s[0] * e, vc_s[1] * e, vc_s[2] * e, lens, src, dst, rb),
                  "kv_move_row");
  DSPARK_CUDA_TRY(launch_ex(kv_move_lens_kernel, dim3(1), dim3(32), 0, s, 1, true, lens, src, dst),
                  "kv_move_row lens");
  return DSPARK_OK;
}

int argmax(const bf16* logits, int64_t ld, int R, int V, int32_t* tt, cudaStream_t s) {
  if (R <= 0 || V <= 0) return fail(DSPARK_ERR_ARG, "argmax: empty shape");
  if ((reinterpret_cast<uintptr_t>(logits) & 15) || (ld & 7))
    return fail(DSPARK_ERR_UNSUPPORTED, "argmax: logits rows must be 16-byte aligned");
  DSPARK_CUDA_TRY(launch_ex(argmax_kernel, dim3(R), dim3(1024), 0, s, 1, true, logits, ld, V, tt),
                  "argmax");
  return DSPARK_OK;
}

int accept(const int32_t* tt, const int32_t* ids, const int32_t* cu, int B, int32_t* n_accept,
           int32_t* next_tok, int32_t* lens, cudaStream_t s) {
  if (B <= 0) return DSPARK_OK;
  DSPARK_CUDA_TRY(launch_ex(accept_kernel, dim3((B + 127) / 128), dim3(128), 0, s, 1, true, tt, ids,
                            cu, B, n_accept, next_tok, lens),
                  "accept");
  return DSPARK_OK;
}

int pack_ragged(const int32_t* block_len, const int32_t* kv_len, const int64_t* slot_off,
                const int32_t* ids_pad, int t_max, int B, int r_max, int32_t* cu, int32_t* row_pos,
                int64_t* row_kv, int32_t* row_req, int32_t* ids, int32_t* kv_len_new,
                cudaStream_t s) {
  if (B < 0 || B > 4096) return fail(DSPARK_ERR_UNSUPPORTED, "pack_ragged: B=%d outside 0..4096", B);
  DSPARK_CUDA_TRY(launch_ex(pack_kernel, dim3(1), dim3(1024), 0, s, 1, true, block_len, kv_len,
                            slot_off, ids_pad, t_max, B, r_max, cu, row_pos, row_kv, row_req, ids,
                            kv_len_new),
                  "pack_ragged");
  return DSPARK_OK;
}

int batch_mask(const int32_t* off, int B, int T, int Lcur, uint8_t* mask, cudaStream_t s) {
  const int64_t total = int64_t(B) * T * Lcur;
  if (total <= 0) return DSPARK_OK;
  const int blocks = int(std::min<int64_t>(4096, (total + 255) / 256));
  DSPARK_CUDA_TRY(launch_ex(batch_mask_kernel, dim3(blocks), dim3(256), 0, s, 1, false, off, B, T,
                            Lcur, mask),
                  "batch_mask");
  return DSPARK_OK;
}

int embed(const int32_t* ids, int M, const uint32_t* wq, const bf16* sc, const bf16* bi, int H,
          int V, int bits, bf16* h, float* ssq, cudaStream_t s) {
  if (H % 64) return fail(DSPARK_ERR_UNSUPPORTED, "embed: hidden %% 64 != 0");
  if (V <= 0 || M <= 0) return fail(DSPARK_ERR_ARG, "embed: V=%d M=%d", V, M);
  if (bits == 4)
    DSPARK_CUDA_TRY(launch_ex(embed_kernel<4>, dim3(M), dim3(256), 0, s, 1, true, ids, wq, sc, bi,
                              H, V, h, ssq),
                    "embed");
  else if (bits == 8)
    DSPARK_CUDA_TRY(launch_ex(embed_kernel<8>, dim3(M), dim3(256), 0, s, 1, true, ids, wq, sc, bi,
                              H, V, h, ssq),
                    "embed");
  else
    return fail(DSPARK_ERR_UNSUPPORTED, "embed: bits %d", bits);
  return DSPARK_OK;
}

int rmsnorm(const bf16* x, int64_t ldx, int M, int H, const bf16* w, float eps, bf16* out,
            int64_t ldo, cudaStream_t s) {
  DSPARK_CUDA_TRY(launch_ex(rmsnorm_kernel, dim3(M), dim3(256), 0, s, 1, true, x, ldx, H, w, eps,
                            out, ldo),
                  "rmsnorm");
  return DSPARK_OK;
}

int verify_prepare(int32_t* len, int R, int32_t* row_pos, int64_t* row_kv, int32_t* kv_len,
                   int32_t* row_start, int32_t* q_len, int64_t* kv_off, cudaStream_t s) {
  if (R <= 0 || R > 1024) return fail(DSPARK_ERR_ARG, "verify_prepare: R=%d", R);
  DSPARK_CUDA_TRY(launch_ex(verify_prepare_kernel, dim3(1), dim3(std::max(32, (R + 31) / 32 * 32)),
                            0, s, 1, true, len, R, row_pos, row_kv, kv_len, row_start, q_len,
                            kv_off),
                  "verify_prepare");
  return DSPARK_OK;
}

int fill_inv_freq(float* inv_freq, int head_dim, float theta, cudaStream_t s) {
  const int half = head_dim / 2;
  DSPARK_CUDA_TRY(launch_ex(inv_freq_kernel, dim3(1), dim3((half + 31) / 32 * 32), 0, s, 1, false,
                            inv_freq, half, std::log2(theta)),
                  "inv_freq");
  return DSPARK_OK;
}

}  // namespace ops
}  // namespace dspark
