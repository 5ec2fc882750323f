// Internal interface of the KV / accept / packing / glue kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dspark {
namespace ops {

typedef __nv_bfloat16 bf16;

struct KvAppend {
  const void* kn;
  int64_t kn_s[3];  // element strides {batch, head, row}
  const void* vn;
  int64_t vn_s[3];
  void* kc;
  int64_t kc_s[3];
  void* vc;
  int64_t vc_s[3];
  int32_t* lens;
  int B, H, T, D, cap;
  int esize = 2;    // bytes per element
};

int kv_append(const KvAppend& a, cudaStream_t s);
int kv_rollback(int32_t* lens, const int32_t* n_rej, int B, cudaStream_t s);
int kv_move_row(void* kc, const int64_t* kc_s, void* vc, const int64_t* vc_s, int32_t* lens,
                int src, int dst, int H, int D, int esize, int max_len, cudaStream_t s);
int argmax(const bf16* logits, int64_t ld, int R, int V, int32_t* tt, cudaStream_t s);
int accept(const int32_t* tt, const int32_t* ids, const int32_t* cu, int B, int32_t* n_accept,
           int32_t* next_tok, int32_t* lens, cudaStream_t s);
int pack_ragged(const int32_t* block_len, const int32_t* kv_len, const int64_t* slot_off,
                const int32_t* ids_pad, int t_max, int B, int r_max, int32_t* cu, int32_t* row_pos,
                int64_t* row_kv, int32_t* row_req, int32_t* ids, int32_t* kv_len_new,
                cudaStream_t s);
int batch_mask(const int32_t* off, int B, int T, int Lcur, uint8_t* mask, cudaStream_t s);
int embed(const int32_t* ids, int M, const uint32_t* wq, const bf16* sc, const bf16* bi, int H,
          int V, int bits, bf16* h, float* ssq, cudaStream_t s);
int rmsnorm(const bf16* x, int64_t ldx, int M, int H, const bf16* w, float eps, bf16* out,
            int64_t ldo, cudaStream_t s);
int verify_prepare(int32_t* len, int R, int32_t* row_pos, int64_t* row_kv, int32_t* kv_len,
                   int32_t* row_start, int32_t* q_len, int64_t* kv_off, cudaStream_t s);
int fill_inv_freq(float* inv_freq, int head_dim, float theta, cudaStream_t s);

}  // namespace ops
}  // namespace dspark
