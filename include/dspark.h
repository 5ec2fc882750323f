/*
 * dspark.h — C ABI of the B200 (sm_100a) speculative-decoding verify path.
 *
 * Every entry point takes plain device pointers (caller-owned, written in place), sizes and
 * a cudaStream_t passed as void*, launches asynchronously on that stream and returns an int
 * status: DSPARK_OK, or an error code with a message in dspark_last_error(). Nothing is
 * allocated per call; scratch space, where a launch needs any, is passed in. There is no
 * CPU fallback: an unsupported shape is an error.
 *
 * bf16 tensors are passed as void* (2-byte elements); the weight format is MLX's affine
 * quantization with group size 64: packed uint32 [N, K*bits/32] LSB-first, bf16 scales and
 * biases [N, K/64], w = scale*q + bias.
 */
#ifndef DSPARK_H_
#define DSPARK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DSPARK_OK 0
#define DSPARK_ERR_ARG 1          /* invalid argument */
#define DSPARK_ERR_UNSUPPORTED 2  /* shape / alignment / format the kernels do not serve */
#define DSPARK_ERR_CUDA 3         /* CUDA runtime error (launch, attribute, ...) */
#define DSPARK_ERR_TIMEOUT 4      /* a bounded wait ran out (device status word set) */
#define DSPARK_ERR_NOT_INIT 5     /* dspark_init() was not called for this device */

/* Library version (major*10000 + minor*100 + patch). */
int dspark_version(void);

/* Message for the last error returned on this host thread ("" when none). */
const char* dspark_last_error(void);

/* One-time per-device set-up (allocates the device status word). Call before any launch on
 * `device` and before capturing launches into a CUDA graph. */
int dspark_init(int device);

/* Read (and optionally clear) the device status word: 0, or the code of the first bounded
 * wait that ran out on that device. Synchronizes the device. */
int dspark_device_status(int device, int* code, int clear);

/* Bound of every kernel wait on `device` (a stage, a cluster peer, a peer GPU's flag), in
 * nanoseconds; 0 restores the built-in 2 s. A wait that runs out records its code in the status
 * word and the kernel drains without further waits. Library extension for failure detection (the
 * reference has no device waits: MLX raises on the host). Synchronizes the device. */
int dspark_set_wait_limit_ns(int device, uint64_t ns);

/* Number of streaming multiprocessors of `device` (launch planning). */
int dspark_sm_count(int device);

/* Kernel launches this library has issued since it was loaded (all devices; launches
 * captured into a CUDA graph count once, at capture). */
long long dspark_launch_count(void);

/* ------------------------------------------------------------------------------------ K1 */

/* out[M,N] = x[M,K] . dequant(W)^T, fp32 accumulation, bf16 result, 1 <= M <= 32.
 * Replaces skinny_qmm.qmm(x2, weight, scales, biases, bits)
 * (src/mlx_dspark/skinny_qmm.py:239) and mx.quantized_matmul(x, w, scales, biases,
 * transpose=True, group_size=64, bits) at the call site skinny_qmm.call
 * (src/mlx_dspark/skinny_qmm.py:249) reached from small_m_qmm._mma_call
 * (src/mlx_dspark/small_m_qmm.py:71). Requires K % 64 == 0, N % 8 == 0, group == 64,
 * bits in {4, 8}, x 16-byte aligned, contiguous rows. */
int dspark_qmm(const void* x, int M, int K, const uint32_t* wq, const void* scales,
               const void* biases, int N, int bits, int group, void* out, void* stream);

/* dspark_qmm with row strides (elements) and an optional bf16 bias [N] added after the
 * product in bf16 (QuantizedLinear's bias, src/mlx_dspark/skinny_qmm.py:263-264). */
int dspark_qmm_ex(const void* x, int64_t ldx, int M, int K, const uint32_t* wq,
                  const void* scales, const void* biases, const void* bias, int N, int bits,
                  int group, void* out, int64_t ldo, void* stream);

/* Epilogues of dspark_qmm_fused. */
#define DSPARK_EPI_PLAIN 0   /* out = bf16(x . W^T) (+ bias) */
#define DSPARK_EPI_RESID 1   /* out = bf16(bf16(x . W^T) + resid); ssq_out[tile][m] = sum out^2 */
#define DSPARK_EPI_SWIGLU 2  /* rows gate/up interleaved in blocks of 32: out = silu(g) * u */
#define DSPARK_EPI_QKROPE 3  /* Qwen3 q/k RMSNorm + rotate-half RoPE; q to q_out, k/v to caches */

/* One quantized matmul with the verify forward's fused prologue / epilogues (no single
 * reference counterpart: it is one QuantizedLinear call of mlx-lm's Qwen3 layer, reached from
 * src/mlx_dspark/target.py:208-221, with its neighbouring norm / residual / SwiGLU / RoPE
 * fused): the building block of a layer, e.g. for a forward whose projections are column-sharded over GPUs (each
 * rank runs its shard and all-gathers). An optional RMSNorm prologue scales x by
 * rsqrt(mean of the row's squares + eps) * norm_w, the mean taken from ssq_n partial sums
 * ssq_in[e * ssq_stride + m]. x rows may be segmented (x_seg > 0): element k of row m at
 * x + (k / x_seg) * x_seg_stride + m * ldx + k % x_seg, the [P, M, K/P] layout an all-gather of
 * column shards produces. M <= 32. Same numerics as dspark_verify_forward's projections. */
typedef struct {
  const void* x;
  int64_t ldx, x_seg, x_seg_stride;
  int M, K, N, bits;
  const uint32_t* wq;
  const void* scales;
  const void* biases;
  void* out;
  int64_t ldo;
  int epilogue;                     /* DSPARK_EPI_* */
  const void* bias;                 /* PLAIN: optional bf16 [N] */
  const void* norm_w;               /* optional RMSNorm prologue weight [K] */
  const float* ssq_in;
  int ssq_n, ssq_stride;
  float eps;
  const void* resid;                /* RESID */
  int64_t ldr;
  float* ssq_out;
  int n_act;                        /* SWIGLU: activation columns (N / 2) */
  int hq, hk;                       /* QKROPE: local q / kv heads (head_dim 128) */
  const void* q_norm;
  const void* k_norm;
  const float* inv_freq;            /* [64] from dspark_rope_inv_freq */
  void* q_out;
  int64_t ldq;
  void* k_cache;
  void* v_cache;
  int64_t k_sh, k_ss, v_sh, v_ss;
  int kv_cap;
  const int32_t* row_pos;           /* [M] absolute positions */
  const int64_t* row_kv;            /* [M] cache slot offsets (elements), or NULL */
  int ssq_seg;                      /* > 0: entry e of ssq_in at (e / ssq_seg) * ssq_seg_stride */
  int64_t ssq_seg_stride;           /*      + (e % ssq_seg) * ssq_stride (gathered statistics) */
  /* Tensor-parallel gathers fused into the projections (K % 512 == 0, not with
   * DSPARK_QMM_ST_TC). Peer stores (RESID / SWIGLU): every output element, and every RESID
   * statistic, is also stored at its address + peer_delta[s] for each rank s < peer_world
   * (peer_delta[own rank] = 0: the buffers sit at one offset in every rank's IPC arena, see
   * dspark_ipc_alloc). After each output tile the writing CTA adds the number of elements it
   * stored to the uint32 at peer_flag + peer_delta[s] (system-scope release). peer_world = 0: off. */
  int peer_world;
  int64_t peer_delta[8];
  uint32_t* peer_flag;
  /* Wait (before x is read) until wait_flag[s] >= wait_state[0] + wait_elems for every source
   * s < wait_world (bounded, ~2 s); the launch's last CTA then advances wait_state[0] by
   * wait_elems (wait_state[1] counts the launch's finished CTAs). wait_flag = NULL: no wait. */
  const uint32_t* wait_flag;
  int wait_world;
  uint32_t wait_elems;
  uint32_t* wait_state;
} dspark_qmm_args;

int dspark_qmm_fused(const dspark_qmm_args* a, void* stream);

/* Wide-M product out[M, N] = bf16(x[M, K] . dequant(W)^T) for any number of rows (prefill-width
 * calls, the batch engine's packed rows): the weights are dequantized once per 128-row tile into
 * tensor memory (w = scale * q + bias rounded to bf16) and multiplied with 256 x rows per
 * tcgen05 MMA, fp32 accumulation. Replaces wide_gemm's x @ mx.dequantize(w).T
 * (src/mlx_dspark/wide_gemm.py:1-30, the patched call at :177-193). Requires K % 512 == 0,
 * bits in {4, 8}, group 64, x / weights / scales / biases 16-byte aligned, ldx % 8 == 0. */
int dspark_qmm_wide(const void* x, int64_t ldx, int M, int K, const uint32_t* wq,
                    const void* scales, const void* biases, int N, int bits, void* out,
                    int64_t ldo, void* stream);

/* Scratch bytes a wide projection of dspark_verify_forward needs: the normed x [M, K] when
 * `norm`, and the bf16 product [M, N] when the epilogue is not DSPARK_EPI_PLAIN. */
size_t dspark_qmm_wide_workspace(int M, int K, int N, int epilogue, int norm);

/* RoPE frequencies theta^(-2i/head_dim), i < head_dim / 2, as the fused epilogue uses them. */
int dspark_rope_inv_freq(float* inv_freq, int head_dim, float theta, void* stream);

/* Launch geometry the QMM uses for [N, K] at `bits` for 1-16 rows: tile width, split-K
 * cluster size, k per split, pipeline depth. The plan is fixed within each row class (1-16 rows
 * and 17-32 rows), so inside a class a row's result never depends on how many rows ride with it.
 * Mirrors skinny_qmm.plan/geometry (src/mlx_dspark/skinny_qmm.py:214-236). */
int dspark_qmm_plan(int N, int K, int bits, int* tile_n, int* split_k, int* k_slice,
                    int* stages);

/* The plan dspark_qmm runs for `rows` (1..32) rows: out[0] tile width, out[1] split-K cluster
 * size, out[2] k per split, out[3] pipeline depth, out[4] persistent clusters (0: one per tile),
 * out[5] launches (2 when a 17-32-row call runs as two 16-row launches), out[6] engine (2:
 * streaming, 1: tcgen05 / tensor memory, 0: per-tile CTAs). Same plan source as
 * dspark_qmm_plan. */
int dspark_qmm_plan_rows(int N, int K, int bits, int rows, int out[7]);

/* ------------------------------------------------------------------------------------ K2 */

/* Multi-row GQA verify attention, out = softmax(scale * q.k^T + mask) . v.
 * Replaces multirow_attn.multirow_sdpa(q, k, v, scale=, causal=, tree_anc=)
 * (src/mlx_dspark/multirow_attn.py:223), i.e. mx.fast.scaled_dot_product_attention with
 * mask=None/"causal" for few-row blocks (patched at src/mlx_dspark/multirow_attn.py:338).
 * Shapes: q [B, Hq, qL, D], k/v [B, Hk, L, D] (any strides with D contiguous, cache views
 * allowed), out [B, Hq, qL, D]; strides are element strides {batch, head, row}. Causal rule:
 * row i sees keys <= L - qL + i. tree_anc (uint32 [B*qL], optional) switches to the
 * tree-verify rule: every key < L - qL, and key L - qL + j iff bit j of anc[i]
 * (src/mlx_dspark/multirow_attn.py:184-195). kv_len (device int32 [B], optional) gives a
 * per-row key count <= L. D in {64, 128, 256}. bf16 tensors (dspark_verify_attn_dt takes the
 * element type). workspace may be NULL when dspark_verify_attn_workspace() returns 0 for the
 * shape. */
int dspark_verify_attn(const void* q, const int64_t q_strides[3], const void* k,
                       const int64_t k_strides[3], const void* v, const int64_t v_strides[3],
                       int B, int Hq, int Hk, int qL, int D, int L, const int32_t* kv_len,
                       float scale, int causal, const uint32_t* tree_anc, void* out,
                       const int64_t o_strides[3], void* workspace, size_t ws_bytes,
                       void* stream);

/* Element types of dspark_verify_attn_dt. */
#define DSPARK_DTYPE_BF16 0
#define DSPARK_DTYPE_F16 1

/* dspark_verify_attn for q/k/v/out of element type `dtype` (bf16 or fp16, the two input types
 * multirow_sdpa serves, src/mlx_dspark/multirow_attn.py:304; the probabilities are rounded
 * to that type for P.V as the reference kernel does, :136-140). Same shapes and rules. */
int dspark_verify_attn_dt(int dtype, const void* q, const int64_t q_strides[3], const void* k,
                          const int64_t k_strides[3], const void* v, const int64_t v_strides[3],
                          int B, int Hq, int Hk, int qL, int D, int L, const int32_t* kv_len,
                          float scale, int causal, const uint32_t* tree_anc, void* out,
                          const int64_t o_strides[3], void* workspace, size_t ws_bytes,
                          void* stream);

/* dspark_verify_attn for callers that cannot allocate device memory (no workspace argument).
 * This entry point has no counterpart in the reference: it exists for code that is being
 * captured into a CUDA graph (where cudaMalloc is not allowed), for plugins whose host runtime
 * owns all device memory and passes only input and output buffers, and for paths that must not
 * let an allocation or a cudaFree stall the device. Its scratch is a static 4 MiB device array
 * per GPU (held until exit); shapes whose workspace (dspark_verify_attn_workspace) exceeds it
 * fail with DSPARK_ERR_UNSUPPORTED. The first call on a device looks up that array's device
 * address, so make it before any stream capture. The stream must belong to the current device
 * (a stream of another device is DSPARK_ERR_ARG). Calls share the array: calls that overlap on
 * the GPU race. Nothing is allocated and nothing needs clearing between calls. */
int dspark_verify_attn_noalloc(const void* q, const int64_t q_strides[3], const void* k,
                               const int64_t k_strides[3], const void* v,
                               const int64_t v_strides[3], int B, int Hq, int Hk, int qL, int D,
                               int L, const int32_t* kv_len, float scale, int causal,
                               const uint32_t* tree_anc, void* out, const int64_t o_strides[3],
                               void* stream);

/* Launch geometry of dspark_verify_attn for a shape (mirrors multirow_attn.plan,
 * src/mlx_dspark/multirow_attn.py:204-220): out[0] 16-row tiles per CTA, out[1] warps
 * splitting each K/V tile, out[2] row groups, out[3] key splits merged in a cluster, out[4]
 * cluster groups merged through the workspace, out[5] keys per split. */
int dspark_verify_attn_plan(int B, int Hq, int Hk, int qL, int D, int L, int out[6]);

/* Bytes of workspace dspark_verify_attn needs for this shape (0 for most shapes). */
size_t dspark_verify_attn_workspace(int B, int Hq, int Hk, int qL, int D, int L);

/* Ragged form used by the batch engine: request b owns q/out rows starting at row_start[b]
 * (element offset row_start[b]*q_si / *o_si) with q_len[b] rows, and kv_len[b] keys at
 * element offset kv_off[b] of the K/V pools. Max sizes qL_max / L_max bound the launch. */
int dspark_verify_attn_ragged(const void* q, int64_t q_sh, int64_t q_si, const void* k,
                              int64_t k_sh, int64_t k_ss, const void* v, int64_t v_sh,
                              int64_t v_ss, const int32_t* row_start, const int32_t* q_len,
                              const int64_t* kv_off, const int32_t* kv_len, int B, int Hq,
                              int Hk, int qL_max, int D, int L_max, float scale, void* out,
                              int64_t o_sh, int64_t o_si, void* workspace, size_t ws_bytes,
                              void* stream);

/* ------------------------------------------------------------------------------------ K3 */

/* Append T new rows per batch row at that row's current length and advance it:
 * cache[b, h, lens[b] + t, :] = new[b, h, t, :]; lens[b] += T. Rows that would pass `cap`
 * are not written (the device status word records it). Replaces the per-row write loop of
 * BatchCache.update_and_fetch (src/mlx_dspark/batch_engine.py:193-208). Strides in
 * elements {batch, head, row}; D contiguous; elem_size bytes per element (rows of
 * D*elem_size bytes, a multiple of 16, 16-byte aligned). */
int dspark_kv_append(const void* k_new, const int64_t kn_strides[3], const void* v_new,
                     const int64_t vn_strides[3], void* k_cache, const int64_t kc_strides[3],
                     void* v_cache, const int64_t vc_strides[3], int32_t* lens, int B, int H,
                     int T, int D, int elem_size, int cap, void* stream);

/* Quantized KV cache (the reference's kv_bits, src/mlx_dspark/target.py:166-185: mlx-lm's
 * QuantizedKVCache with group size 64): keys and values stored MLX-affine quantized per group of
 * 64 along head_dim, packed uint32 words [.., L, D*bits/32] (LSB-first, the weight format) with
 * bf16 scales and biases [.., L, D/64], value = scale * q + bias. K and V share strides. */
typedef struct {
  uint32_t* kq;            /* key codes */
  void* ks;                /* key scales (bf16) */
  void* kb;                /* key biases (bf16) */
  uint32_t* vq;
  void* vs;
  void* vb;
  int64_t q_strides[3];    /* element strides {batch, head, row} of the code words (uint32) */
  int64_t s_strides[3];    /* element strides {batch, head, row} of the scales / biases */
  int bits;                /* 4 or 8 */
} dspark_qkv;

/* dspark_kv_append into a quantized cache: each new K/V row (bf16, strides {b, h, t}) is
 * quantized per group of 64 (scale = max((max - min) / (2^bits - 1), 1e-8) in fp32, bias = min,
 * q = round-half-even((x - bias) / scale) clamped, scale and bias stored as bf16) at row
 * lens[b] + t, then lens[b] += T. Replaces QuantizedKVCache.update_and_fetch's
 * mx.quantize of the block (src/mlx_dspark/target.py:182). D in {64, 128}. */
int dspark_kv_append_q(const void* k_new, const int64_t kn_strides[3], const void* v_new,
                       const int64_t vn_strides[3], const dspark_qkv* cache, int32_t* lens, int B,
                       int H, int T, int D, int cap, void* stream);

/* dspark_verify_attn over a quantized cache (mlx-lm's quantized_scaled_dot_product_attention
 * route for QuantizedKVCache layers): the K/V tiles are dequantized (scale * q + bias, rounded to
 * bf16) in shared memory and the same verify attention runs on them; q / out bf16 as in
 * dspark_verify_attn. D in {64, 128}, bits in {4, 8}. */
int dspark_verify_attn_q(const void* q, const int64_t q_strides[3], const dspark_qkv* kv, int B,
                         int Hq, int Hk, int qL, int D, int L, const int32_t* kv_len, float scale,
                         int causal, void* out, const int64_t o_strides[3], void* workspace,
                         size_t ws_bytes, void* stream);

/* In-place rollback: lens[b] = max(0, lens[b] - n_rejected[b]) on the device. Metadata only;
 * the next append overwrites the tail. Replaces KVCache.trim / Target.rollback
 * (src/mlx_dspark/target.py:679-698) and BatchCache.trim (src/mlx_dspark/batch_engine.py:220-224). */
int dspark_kv_rollback(int32_t* lens, const int32_t* n_rejected, int B, void* stream);

/* Copy row src's live K/V columns onto row dst and vacate src (lens[dst] = lens[src],
 * lens[src] = 0). Replaces BatchCache.move_row (src/mlx_dspark/batch_engine.py:177-185). */
int dspark_kv_move_row(void* k_cache, const int64_t kc_strides[3], void* v_cache,
                       const int64_t vc_strides[3], int32_t* lens, int src, int dst, int H,
                       int D, int elem_size, int max_len, void* stream);

/* --------------------------------------------------------------------- accept / argmax */

/* tt[r] = argmax(logits[r, :V]) for R rows (first index on ties), logits row stride ld. */
int dspark_argmax(const void* logits, int64_t ld, int R, int V, int32_t* tt, void* stream);

/* Greedy accept over ragged verify blocks, fused with the KV rollback.
 * Request b's block is rows cu_rows[b] .. cu_rows[b+1]-1 of `ids` ([pending, drafts...]) and
 * `tt` (argmax per row). n_accept[b] = length of the leading run of drafts equal to the
 * target's argmax (cumprod(drafts == tt[:cap]).sum(), src/mlx_dspark/generate.py:1548-1550,
 * batched src/mlx_dspark/batch_engine.py:684-686); next_tok[b] = tt[cu_rows[b] + n] (the
 * bonus token); if lens != NULL, lens[b] -= cap - n (the rollback of the rejected tail,
 * src/mlx_dspark/batch_engine.py:692-705). A request with no rows this step (an idle slot)
 * gets n_accept = 0, next_tok = -1 and keeps its length. */
int dspark_accept(const int32_t* tt, const int32_t* ids, const int32_t* cu_rows, int B,
                  int32_t* n_accept, int32_t* next_tok, int32_t* lens, void* stream);

/* ------------------------------------------------------------------------------------ K4 */

/* Ragged request packing for one batched verify step, built on the device.
 * Inputs per active request b < B: block_len[b] (cap_b + 1 rows), kv_len[b] (tokens cached
 * before the step), slot_off[b] (element offset of the request's K/V slot in the pools),
 * ids_pad [B, t_max] ([pending, drafts...], row stride t_max).
 * Outputs: cu_rows [B+1] (prefix sum of block_len), row_pos [R] (absolute position of each
 * packed row = kv_len[b] + i), row_kv [R] (= slot_off of the row's request), row_req [R],
 * ids [R] (packed tokens), kv_len_new [B] (= kv_len + block_len: keys visible to the
 * step's attention), with R = cu_rows[B] <= r_max. Rows r >= R up to r_max are filled
 * with a harmless copy of row 0's metadata. Replaces the host loops of SpecSlots.step /
 * build_batch_mask / BatchCache.update_and_fetch (src/mlx_dspark/batch_engine.py:635-708,
 * :231-239, :193-208). */
int dspark_pack_ragged(const int32_t* block_len, const int32_t* kv_len, const int64_t* slot_off,
                       const int32_t* ids_pad, int t_max, int B, int r_max, int32_t* cu_rows,
                       int32_t* row_pos, int64_t* row_kv, int32_t* row_req, int32_t* ids,
                       int32_t* kv_len_new, void* stream);

/* Boolean mask [B, 1, T, Lcur] (uint8) of build_batch_mask (src/mlx_dspark/batch_engine.py:
 * 231-239): mask[b, 0, i, j] = j <= offsets[b] + i, Lcur = max(offsets) + T. For checking
 * the packing against the reference's dense formulation; the kernels never build it. */
int dspark_batch_mask(const int32_t* offsets, int B, int T, int Lcur, uint8_t* mask,
                      void* stream);

/* --------------------------------------------------------------------- forward glue */

/* h[m] = dequant(embedding[ids[m]]) (MLX QuantizedEmbedding, 4/8-bit g64) in bf16;
 * ssq[m] (optional) = sum(h[m]^2) in fp32 over the bf16 values. */
int dspark_embed(const int32_t* ids, int M, const uint32_t* wq, const void* scales,
                 const void* biases, int V, int H, int bits, void* h, float* ssq, void* stream);

/* out = x * rsqrt(mean(x^2) + eps) * w  (mx.fast.rms_norm), fp32 math, bf16 out. */
int dspark_rmsnorm(const void* x, int64_t ldx, int M, int H, const void* w, float eps,
                   void* out, int64_t ldo, void* stream);

/* Dense Qwen3-style target (random-init or loaded) described by device pointers. */
typedef struct {
  const uint32_t* wq;
  const void* scales;
  const void* biases;
  int N, K, bits;
} dspark_qweight;

typedef struct {
  dspark_qweight qkv;      /* rows [q heads | k heads | v heads], K = hidden */
  dspark_qweight o;        /* N = hidden, K = Hq*D */
  dspark_qweight gate_up;  /* rows interleaved in blocks of 32: gate 32, up 32, ... */
  dspark_qweight down;     /* N = hidden, K = intermediate */
  const void* in_norm;     /* [hidden] */
  const void* post_norm;   /* [hidden] */
  const void* q_norm;      /* [head_dim] */
  const void* k_norm;      /* [head_dim] */
  void* k_cache;           /* layer's K pool: element (h, pos, d) at h*k_sh + pos*k_ss + d */
  void* v_cache;
} dspark_layer;

typedef struct {
  int n_layers, hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab;
  float rms_eps, rope_theta;
  dspark_qweight embed;    /* [vocab, hidden] quantized embedding */
  dspark_qweight lm_head;  /* [vocab, hidden] */
  const void* final_norm;  /* [hidden] */
  const dspark_layer* layers;  /* host array [n_layers] */
  int64_t k_sh, k_ss, v_sh, v_ss;  /* cache strides (elements) */
  int kv_cap;              /* positions per request slot */
} dspark_model;

/* Caller-owned device buffers for one verify forward of up to rows_cap packed rows (h, xq,
 * attn, act and the logits hold rows_cap rows; the statistics buffers 1024 * rows_cap floats). */
typedef struct {
  void* h;          /* bf16 [r_max, hidden] residual stream */
  void* xq;         /* bf16 [r_max, n_heads*head_dim] roped queries */
  void* attn;       /* bf16 [r_max, n_heads*head_dim] attention output */
  void* act;        /* bf16 [r_max, intermediate] SwiGLU output */
  float* ssq_a;     /* fp32 [1024 * rows_cap] RMSNorm partial statistics */
  float* ssq_b;     /* fp32 [1024 * rows_cap] */
  float* inv_freq;  /* fp32 [head_dim/2] RoPE frequencies (filled by the forward) */
  int32_t* row_pos; /* int32 [r_max] absolute positions */
  int64_t* row_kv;  /* int64 [r_max] element offset of each row's cache slot */
  int32_t* kv_len;  /* int32 [B] keys visible per request (after the append) */
  int32_t* row_start;  /* int32 [B] first packed row of each request */
  int32_t* q_len;      /* int32 [B] rows per request */
  int64_t* kv_off;     /* int64 [B] cache slot offset per request */
  void* attn_ws;    /* attention workspace (may be NULL) */
  size_t attn_ws_bytes;
  int rows_cap;     /* rows the buffers hold (0: 32) */
  void* wide_ws;    /* scratch of the wide-M projections (NULL: 32-row launches only) */
  size_t wide_ws_bytes;  /* >= the largest dspark_qmm_wide_workspace of the model's projections */
} dspark_fwd_buffers;

/* One verify forward (Target.verify -> _body_mlxlm + head, src/mlx_dspark/target.py:642,
 * :208-221; batched_forward src/mlx_dspark/batch_engine.py:245-276) over R packed rows of B
 * requests: embed -> n_layers x [RMSNorm, fused QKV QMM + q/k-norm + RoPE + cache write,
 * verify attention, O QMM + residual, RMSNorm, gate/up QMM + SwiGLU, down QMM + residual]
 * -> RMSNorm -> lm_head QMM -> logits [R, vocab] (row stride ld_logits).
 * The packing arrays in `buf` (row_pos, row_kv, kv_len, row_start, q_len, kv_off) must be
 * filled for the step (dspark_pack_ragged, or dspark_verify_prepare for one request).
 * L_max / qL_max bound the requests' key counts / block rows (qL_max <= 32). R <= rows_cap:
 * a step of many requests (the batch engine) runs every projection over all R rows at once in
 * the wide-M engine (RMSNorm applied to x, tcgen05 product, fused epilogue on the product) when
 * R >= 64 and buf->wide_ws holds the scratch, else in launches of 32 rows (each re-reads the
 * weights); the attention runs over all requests at once. */
int dspark_verify_forward(const dspark_model* m, const dspark_fwd_buffers* buf,
                          const int32_t* ids, int R, int B, int qL_max, int L_max,
                          void* logits, int64_t ld_logits, void* stream);

/* Single-request packing for dspark_verify_forward: with L0 = *len (device int32, tokens
 * cached before the step): row_pos[m] = L0 + m, row_kv[m] = 0, kv_len[0] = L0 + R,
 * row_start[0] = 0, q_len[0] = R, kv_off[0] = 0, and *len = L0 + R (the forward appends the
 * block's K/V; dspark_accept then trims the rejected tail). */
int dspark_verify_prepare(int32_t* len, int R, const dspark_fwd_buffers* buf, void* stream);

/* ---- all-gather over peer memory (tensor-parallel verify) ------------------------------
 * Replaces the NCCL all-gathers between the column-sharded projections (the collective the
 * reference's verify path does not have: it runs 27B targets on one Apple GPU, target.py:208-221;
 * the fused peer-store variant stores a projection's finished rows straight into the peers'
 * arenas from its epilogue). Set-up, once per rank:
 * dspark_ipc_alloc an arena (zero-filled device memory and its IPC handle), share the handles
 * between the ranks' processes, dspark_ipc_open every peer's handle. The arena layout is the
 * caller's, identical on every rank: a flag area (uint32 [8 buffers][8 ranks]), a counter area
 * (uint32 [8][2]) and the gather buffers ([world][seg_bytes] each). */
#define DSPARK_IPC_HANDLE_BYTES 64

int dspark_ipc_alloc(size_t bytes, void** ptr, void* handle /* DSPARK_IPC_HANDLE_BYTES */);
int dspark_ipc_open(const void* handle, void** ptr);
int dspark_ipc_close(void* ptr);
int dspark_ipc_free(void* ptr);

typedef struct dspark_p2p_gather_args {
  void* const* arenas;   /* [world] every rank's arena as mapped in this process (own: local) */
  const void* src;       /* this rank's segment, seg_bytes (16-byte aligned) */
  size_t seg_bytes;      /* multiple of 16 */
  size_t flags_off;      /* byte offsets inside every arena (multiples of 16) */
  size_t count_off;
  size_t dst_off;        /* destination [world][seg_bytes]; segment `rank` receives src */
  int rank, world;       /* world <= 8 */
  int buf;               /* flag / counter slot of the destination buffer, 0..7 */
} dspark_p2p_gather_args;

/* One all-gather: this rank's segment lands in segment `rank` of the destination buffer of every
 * arena; the launch returns (on the stream) once every rank's segment has landed here. All ranks
 * must issue the same gathers in the same order. Waits on peers are bounded (~2 s): a timeout
 * sets the device status word. */
int dspark_p2p_allgather(const dspark_p2p_gather_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DSPARK_H_ */
