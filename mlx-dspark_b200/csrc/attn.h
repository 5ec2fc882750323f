// Internal interface of the multi-row causal GQA verify attention (K2).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dspark {
namespace attn {

struct AttnParams {
  // element (b, h, i, d) of q is q[qoff(b) + h*q_sh + i*q_si + d] with qoff(b) = row_start
  // ? row_start[b]*q_si : b*q_sb; the output o uses the same rule with its own strides.
  const __nv_bfloat16* q = nullptr;
  int64_t q_sb = 0, q_sh = 0, q_si = 0;
  __nv_bfloat16* o = nullptr;
  int64_t o_sb = 0, o_sh = 0, o_si = 0;
  // key j of (b, h): k[kvoff(b) + h*k_sh + j*k_ss + d], kvoff(b) = kv_off ? kv_off[b] : b*k_sb
  const __nv_bfloat16* k = nullptr;
  int64_t k_sb = 0, k_sh = 0, k_ss = 0;
  const __nv_bfloat16* v = nullptr;
  int64_t v_sb = 0, v_sh = 0, v_ss = 0;
  const int32_t* row_start = nullptr;  // [B] ragged packing: first q row of request b
  const int64_t* kv_off = nullptr;     // [B] ragged packing: K/V element offset of request b
  const int32_t* kv_len = nullptr;     // [B] keys visible to request b (else L)
  const int32_t* q_len = nullptr;      // [B] query rows of request b (else qL)
  const uint32_t* tree_anc = nullptr;  // [B*qL] tree-verify ancestor bits (null: causal rule)
  int B = 0, Hq = 0, Hk = 0, qL = 0, D = 0, L = 0;
  float scale_log2 = 0.f;              // scale * log2(e)
  int causal = 1;
  int f16 = 0;                         // q/k/v/o hold fp16 (else bf16); the pointers carry bits
  // launch geometry
  int nrg = 1;        // row groups per (b, kv head)
  int ns = 1;         // key splits merged inside a cluster (cluster size)
  int ng = 1;         // cluster groups merged through the workspace
  int chunk = 64;     // keys per split (multiple of the kernel's key tile, 64 or 32)
  float* ws = nullptr;  // workspace (ng > 1): [B*Hk*nrg][ng][rows][D+2] fp32
  int* status = nullptr;
  // quantized K/V (qbits 4 or 8; k / v unused): codes [.., L, D*qbits/32] uint32 at strides
  // {kq_sb, kq_sh, kq_ss} (words), bf16 scales / biases at {ks_sb, ks_sh, ks_ss} (elements)
  int qbits = 0;
  const uint32_t* kq = nullptr;
  const uint32_t* vq = nullptr;
  const __nv_bfloat16* ksc = nullptr;
  const __nv_bfloat16* kbi = nullptr;
  const __nv_bfloat16* vsc = nullptr;
  const __nv_bfloat16* vbi = nullptr;
  int64_t kq_sb = 0, kq_sh = 0, kq_ss = 0, ks_sb = 0, ks_sh = 0, ks_ss = 0;
};

struct AttnPlan {
  int nrt = 0, ks = 0, nrg = 1, ns = 1, ng = 1, chunk = 64;
};

AttnPlan plan(int B, int Hq, int Hk, int qL, int D, int L);
size_t workspace_bytes(const AttnPlan& pl, int B, int Hk, int D);
int run(AttnParams p, const AttnPlan* plan, cudaStream_t stream);

}  // namespace attn
}  // namespace dspark
