// Device-side building blocks shared by every dspark kernel (sm_100a only).
//
// mbarrier pipelines with bounded waits, TMA (cp.async.bulk.tensor) and bulk copies,
// thread-block-cluster / distributed-shared-memory access, programmatic dependent launch,
// and the legacy-layout bf16 tensor-core MMA used for the small-M contractions.
//
// Every wait on a barrier that another agent (the TMA unit, another warp, another CTA of the
// cluster) completes is bounded by wall-clock time (%globaltimer): when the bound runs out
// the waiting thread records an error code in the library's device status word and carries
// on, so a kernel bug shows up as a host-visible status instead of a hung GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dspark {

typedef __nv_bfloat16 bf16;

// Error codes written into the device status word (see dspark_device_status()).
enum DeviceError : int {
  kErrNone = 0,
  kErrWaitFull = 0x101,      // consumer gave up waiting for a TMA stage
  kErrWaitEmpty = 0x102,     // producer gave up waiting for consumers to free a stage
  kErrWaitKV = 0x103,        // attention consumer gave up waiting for a K/V tile
  kErrWaitKVEmpty = 0x104,   // attention producer gave up waiting for a free K/V slot
  kErrWaitPeer = 0x105,      // a cross-GPU flag wait ran out of time
  kErrWaitCluster = 0x106,   // a CTA gave up waiting for its cluster peers' partial sums
  kErrWaitMma = 0x107,       // a tensor-core completion wait ran out of time
};

// ~2 s: far beyond any legitimate wait inside one kernel launch. The default bound; a process
// can change it per device (dspark_set_wait_limit_ns), which stores the bound in the second
// 8-byte word of the device status block.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// The first ALIGN-byte boundary of a dynamic shared-memory array, formed by pointer arithmetic
// on the array itself, so that the compiler still knows that the pointer (and every pointer
// derived from it) addresses shared memory. A round trip through an integer would give a generic
// pointer, and every C++ access through it a generic load or store: measured at more than twice
// the time of the shared-memory instructions in these kernels.
template <uint32_t ALIGN>
__device__ __forceinline__ uint8_t* smem_align_up(uint8_t* raw) {
  return raw + ((ALIGN - (smem_u32(raw) & (ALIGN - 1u))) & (ALIGN - 1u));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report_error(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// The bound of a wait: the per-device value stored after the status word (bytes 8..15 of the
// status block), or kWaitLimitNs when unset. Read only on a wait's slow path.
__device__ __forceinline__ uint64_t wait_limit_ns(const int* status) {
  if (status == nullptr) return kWaitLimitNs;
  const uint64_t v = *reinterpret_cast<const volatile uint64_t*>(status + 2);
  return v ? v : kWaitLimitNs;
}

// ------------------------------------------------------------------ mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete. Returns false (and records `code`)
// if it has not completed within the wait bound (wait_limit_ns).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = wait_limit_ns(status);
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(a, parity)) return true;
    if (globaltimer_ns() - t0 > limit) {
      report_error(status, code);
      return false;
    }
  }
}

// ------------------------------------------------------------------ TMA / bulk copies

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled tensor load (no multicast) into this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::"
      "cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// 3-D / 4-D tiled TMA loads into this CTA's shared memory, completing on `bar` (no cache hint).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

// Contiguous bulk copy global -> this CTA's shared memory (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 16-byte global -> shared copy through L2 (cp.async.cg); when !valid nothing is read and the
// 16 destination bytes are zero-filled.
__device__ __forceinline__ void cp_async_16_zfill(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}

// Arrive on `bar` once every cp.async this thread issued so far has completed (the arrival
// counts toward the barrier's expected count).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ------------------------------------------------------------------ programmatic dependent launch

// Block until the grids this launch depends on have completed and their writes are visible.
// A no-op when the kernel was launched without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Let the next kernel in the stream start its prologue on free SM slots.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------ clusters / DSMEM

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}

// Split cluster barrier: every thread arrives once (after its CTA's barriers are initialized)
// and waits before its first access to another CTA's shared memory or barriers.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Store to shared memory of a CTA of this cluster (address from mapa_shared); asynchronous
// for the issuing thread, ordered for readers by a later cluster barrier or release/acquire.
__device__ __forceinline__ void st_dsmem_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ void st_dsmem_f4(uint32_t addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}

// Asynchronous stores into the shared memory of a CTA of this cluster (`addr` and `mbar` are
// shared::cluster addresses in that CTA): when the bytes land they count toward the transaction
// count of that CTA's mbarrier, so its waiter needs no fence or arrive from the sender.
__device__ __forceinline__ void st_async_f32(uint32_t addr, float v, uint32_t mbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(
                   addr),
               "f"(v), "r"(mbar)
               : "memory");
}

__device__ __forceinline__ void st_async_v2(uint32_t addr, float a, float b, uint32_t mbar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
          addr),
      "f"(a), "f"(b), "r"(mbar)
      : "memory");
}

// Release (system scope) add to a counter in this or another GPU's memory: the writes this thread
// (and, cumulatively, the threads it synchronised with) made before are visible to whoever
// acquires the new value.
__device__ __forceinline__ void red_add_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// Wait until the monotonic counter *f reaches `target` (wrap-safe); false (and `code` recorded)
// if it has not within the wait bound (wait_limit_ns).
__device__ __forceinline__ bool wait_counter_sys(const uint32_t* f, uint32_t target, int* status,
                                                 int code) {
  if (int32_t(ld_acquire_sys(f) - target) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = wait_limit_ns(status);
  while (int32_t(ld_acquire_sys(f) - target) < 0) {
    if (globaltimer_ns() - t0 > limit) {
      report_error(status, code);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// 16-byte global load through L2 only (data another kernel wrote)
__device__ __forceinline__ uint4 ldcg_v4(const void* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));
}

// 16-byte global load through the read-only path (data no kernel writes while this one runs)
__device__ __forceinline__ uint4 ldg_v4(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ void fence_acq_rel_cluster() {
  asm volatile("fence.acq_rel.cluster;" ::: "memory");
}

// Arrive (release, cluster scope) on the mbarrier at the same shared-memory offset as `bar`
// in CTA `rank` of this cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t* bar, uint32_t rank) {
  const uint32_t remote = mapa_shared(smem_u32(bar), rank);
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// mbar_wait with cluster-scope acquire: for phases completed by arrivals of peer CTAs, whose
// writes to their own shared memory are read afterwards through distributed shared memory.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* status,
                                                  int code) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait_cluster(a, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = wait_limit_ns(status);
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait_cluster(a, parity)) return true;
    if (globaltimer_ns() - t0 > limit) {
      report_error(status, code);
      return false;
    }
  }
}

// (a0, a1) += (b0, b1) * (c0, c1): two independent round-to-nearest fp32 FMAs in one packed
// instruction (sm_100), bit-identical to two fmaf calls.
__device__ __forceinline__ void fma2(float& a0, float& a1, float b0, float b1, float c0, float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\tmov.b64 rc, {%4, %5};\n\t"
      "fma.rn.f32x2 ra, rb, rc, ra;\n\t"
      "mov.b64 {%0, %1}, ra;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

// (a0, a1) *= (b0, b1): two independent round-to-nearest fp32 products in one instruction
__device__ __forceinline__ void mul2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb;\n\t"
      "mov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\t"
      "mul.rn.f32x2 ra, ra, rb;\n\t"
      "mov.b64 {%0, %1}, ra;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1));
}

// ------------------------------------------------------------------ shared-memory vector loads

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// ------------------------------------------------------------------ tensor-core MMA (bf16)

// D[16x8] += A[16x16] * B[16x8], bf16 operands, fp32 accumulate. Register operands only (not
// volatile), so the compiler may interleave it with the shared-memory loads of the next step.
__device__ __forceinline__ void mma_bf16_16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// (a & b) | c in one instruction.
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float bf2f(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

}  // namespace dspark
