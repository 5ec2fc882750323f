// All-gather over peer memory (NVLink / NVSwitch) for the tensor-parallel verify forward.
//
// Each rank allocates one arena with cudaMalloc and shares its CUDA IPC handle; every rank maps
// every peer's arena, so a rank stores straight into its peers' memory. An arena holds, at fixed
// offsets identical on every rank:
//   * flags [kBufs][kMaxRanks] uint32: flag (b, s) counts the blocks of rank s that have
//     finished writing their part of rank s's segment into this arena's buffer b (written by the
//     peers with release atomics, monotonic, never reset);
//   * counts [kBufs][2] uint32: this rank's own round counter of buffer b and the number of
//     this launch's blocks done (touched by this rank only);
//   * the gather buffers, each [world][segment bytes].
//
// One launch per gather: block i copies its share of this rank's segment into segment `rank` of
// buffer b in every arena (16-byte loads and stores), then releases at system scope and adds 1
// to flag (b, rank) of every arena. Block 0 then waits, bounded, until every rank's flag of b has
// reached (round + 1) * blocks: all segments have landed. The last block to finish advances the
// round. All ranks launch the same gathers in the same order with the same block count, so their
// rounds agree; no host epoch is needed and the launch can be captured in a CUDA graph.
//
// Buffer reuse: the forward alternates two buffers per gather kind, so a rank writes into a peer's
// buffer b again only after that peer has signalled a later gather, which it does only after the
// kernels that read b have run (stream order). No TMA multicast and no NVLink multicast objects
// are used: plain peer stores and atomics.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "../../include/dspark.h"
#include "common.cuh"
#include "host_common.h"

namespace dspark {
namespace p2p {

constexpr int kMaxRanks = 8;
constexpr int kBufs = 8;
constexpr int kThreads = 256;
constexpr size_t kChunk = 16384;  // bytes of a segment per block

struct Params {
  char* arena[kMaxRanks];
  const char* src;
  size_t seg;        // segment bytes (multiple of 16)
  size_t flags_off;  // byte offset of the flag area (uint32 [kBufs][kMaxRanks])
  size_t count_off;  // byte offset of the counters (uint32 [kBufs][2])
  size_t dst_off;    // byte offset of the destination buffer [world][seg]
  int rank, world, buf, nblk;
  int* status;
};

__global__ void __launch_bounds__(kThreads) allgather_kernel(const __grid_constant__ Params p) {
  uint32_t* counts = reinterpret_cast<uint32_t*>(p.arena[p.rank] + p.count_off) + p.buf * 2;
  __shared__ uint32_t round;
  if (threadIdx.x == 0) round = __ldcg(&counts[0]);  // read before this block counts itself done
  // this block's share of the segment, in 16-byte words
  const size_t n16 = p.seg / 16;
  const size_t per = (n16 + p.nblk - 1) / p.nblk;
  const size_t i0 = size_t(blockIdx.x) * per, i1 = min(n16, i0 + per);
  const uint4* src = reinterpret_cast<const uint4*>(p.src);
  const size_t dst = p.dst_off + size_t(p.rank) * p.seg;
  for (size_t i = i0 + threadIdx.x; i < i1; i += kThreads) {
    const uint4 v = __ldcg(src + i);
    for (int s = 0; s < p.world; ++s) reinterpret_cast<uint4*>(p.arena[s] + dst)[i] = v;
  }
  __syncthreads();  // this block's stores precede its release below (cumulative)
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int s = 0; s < p.world; ++s)
      red_add_release_sys(reinterpret_cast<uint32_t*>(p.arena[s] + p.flags_off) +
                              p.buf * kMaxRanks + p.rank,
                          1u);
  }
  // completion: block 0 waits until every rank's blocks of this round have landed
  if (blockIdx.x == 0 && threadIdx.x < p.world) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(p.arena[p.rank] + p.flags_off) +
                        p.buf * kMaxRanks + threadIdx.x;
    wait_counter_sys(f, (round + 1u) * uint32_t(p.nblk), p.status, kErrWaitPeer);
  }
  __syncthreads();
  // the last block of this launch advances the round (every block has read it by now)
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&counts[1], 1u) == uint32_t(p.nblk) - 1) {
      counts[1] = 0;
      counts[0] = round + 1;
      __threadfence();
    }
  }
}

}  // namespace p2p
}  // namespace dspark

using namespace dspark;

extern "C" int dspark_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return fail(DSPARK_ERR_ARG, "ipc_alloc: bad arguments");
  void* p = nullptr;
  DSPARK_CUDA_TRY(cudaMalloc(&p, bytes), "ipc_alloc: cudaMalloc");
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(DSPARK_ERR_CUDA, "ipc_alloc: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) <= DSPARK_IPC_HANDLE_BYTES, "handle size");
  std::memset(handle, 0, DSPARK_IPC_HANDLE_BYTES);
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return DSPARK_OK;
}

extern "C" int dspark_ipc_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(DSPARK_ERR_ARG, "ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  DSPARK_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "ipc_open");
  return DSPARK_OK;
}

extern "C" int dspark_ipc_close(void* ptr) {
  DSPARK_CUDA_TRY(cudaIpcCloseMemHandle(ptr), "ipc_close");
  return DSPARK_OK;
}

extern "C" int dspark_ipc_free(void* ptr) {
  DSPARK_CUDA_TRY(cudaFree(ptr), "ipc_free");
  return DSPARK_OK;
}

extern "C" int dspark_p2p_allgather(const dspark_p2p_gather_args* a, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (!a || !a->arenas || !a->src) return fail(DSPARK_ERR_ARG, "p2p_allgather: null arguments");
  if (a->world < 1 || a->world > p2p::kMaxRanks || a->rank < 0 || a->rank >= a->world)
    return fail(DSPARK_ERR_ARG, "p2p_allgather: rank %d of %d (at most %d ranks)", a->rank,
                a->world, p2p::kMaxRanks);
  if (a->buf < 0 || a->buf >= p2p::kBufs)
    return fail(DSPARK_ERR_ARG, "p2p_allgather: buffer %d (0..%d)", a->buf, p2p::kBufs - 1);
  if (a->seg_bytes == 0 || a->seg_bytes % 16 || (a->dst_off | a->flags_off | a->count_off) % 16 ||
      (reinterpret_cast<uintptr_t>(a->src) & 15))
    return fail(DSPARK_ERR_ARG, "p2p_allgather: segments, offsets and source must be 16-byte aligned");
  p2p::Params p;
  std::memset(&p, 0, sizeof(p));
  for (int s = 0; s < a->world; ++s) {
    if (!a->arenas[s] || (reinterpret_cast<uintptr_t>(a->arenas[s]) & 15))
      return fail(DSPARK_ERR_ARG, "p2p_allgather: arena %d missing or unaligned", s);
    p.arena[s] = static_cast<char*>(a->arenas[s]);
  }
  p.src = static_cast<const char*>(a->src);
  p.seg = a->seg_bytes;
  p.flags_off = a->flags_off;
  p.count_off = a->count_off;
  p.dst_off = a->dst_off;
  p.rank = a->rank;
  p.world = a->world;
  p.buf = a->buf;
  // the block count is a function of the segment size only, so every rank uses the same one
  p.nblk = int(std::min<size_t>(148, std::max<size_t>(1, (a->seg_bytes + p2p::kChunk - 1) / p2p::kChunk)));
  p.status = status_word(current_device());
  DSPARK_CUDA_TRY(launch_ex(p2p::allgather_kernel, dim3(p.nblk), dim3(p2p::kThreads), 0, stream, 1,
                            false, p),
                  "p2p_allgather: launch");
  return DSPARK_OK;
}
