// Host-side plumbing shared by the C-ABI entry points: status codes, the per-thread error
// message, the per-device status word, TMA tensor-map encoding and the launch helper that
// attaches cluster / programmatic-dependent-launch attributes.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/dspark.h"

namespace dspark {

// Record a formatted error message for dspark_last_error() and return `code`.
int fail(int code, const char* fmt, ...);

// Turn a CUDA runtime error into DSPARK_ERR_CUDA with a message naming `what`.
int cuda_fail(cudaError_t e, const char* what);

#define DSPARK_CUDA_TRY(expr, what)                 \
  do {                                              \
    cudaError_t _e = (expr);                        \
    if (_e != cudaSuccess) return cuda_fail(_e, what); \
  } while (0)

// Per-device int status word that kernels write on a timed-out wait. Allocated once per
// device by dspark_init(); nullptr when that has not happened yet.
int* status_word(int device);
int current_device();
int sm_count(int device);

// Programmatic dependent launch is used unless DSPARK_PDL=0.
bool pdl_enabled();

// Encode a 2-D tiled tensor map (dim0 innermost). Returns false with an error recorded.
bool encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t dim0,
                    uint64_t dim1, uint64_t stride1_bytes, uint32_t box0, uint32_t box1,
                    CUtensorMapSwizzle swz);

// A rank-`rank` tiled tensor map (dims innermost first, strides of dims 1.. in bytes). Returns
// false, without recording an error, when the driver refuses it: callers fall back to another
// data path.
bool encode_tmap_nd(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                    const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                    CUtensorMapSwizzle swz);

// Integer environment override (tuning knobs); `dflt` when unset.
int env_int(const char* name, int dflt);

// Kernel launches issued through launch_ex since the library was loaded.
void count_launch();

// The value a kernel's function attributes were last configured with on `device` (0: never).
// cudaFuncSetAttribute acts on the current device's context only, so a kernel launched on a
// second device of the same process must be configured there again.
int configured_value(const void* fn, int device);
void set_configured_value(const void* fn, int device, int value);

// Run `setup()` (returning cudaError_t) unless `fn` was configured with at least `value` on the
// current device; record `value` when it succeeds.
template <typename F>
cudaError_t configure_once(const void* fn, int value, F&& setup) {
  const int dev = current_device();
  if (configured_value(fn, dev) >= value) return cudaSuccess;
  const cudaError_t e = setup();
  if (e == cudaSuccess) set_configured_value(fn, dev, value);
  return e;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t stream, int cluster_x, bool pdl, Args&&... args) {
  count_launch();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl && pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace dspark
