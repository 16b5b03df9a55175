// Host-side helpers shared by the C-ABI entry points: status codes, the
// thread-local error string, tensor-map encoding through the driver entry
// point, and per-device properties.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/ldb200.h"

namespace ldb {

void set_last_error(const char* fmt, ...);

// Return `code` after recording a formatted message for ldb_last_error().
int fail(int code, const char* fmt, ...);

// Map a CUDA runtime error to LDB_ERR_CUDA (recording its text), or LDB_OK.
int check_cuda(cudaError_t err, const char* what);

// Number of SMs of the current device (cached per device).
int sm_count();

// Device address of the current device's status word (cached per device).
unsigned int* device_status_ptr();

// Count one kernel launch issued by the library (see ldb_launch_count).
void count_launch(int n = 1);

// Launch `kernel` (every library kernel starts with pdl_begin()) with
// programmatic stream serialization, count it, and map a launch failure to
// LDB_ERR_CUDA with `what` in the message.
template <typename... Params, typename... Args>
int launch_kernel(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                  const char* what, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  return check_cuda(cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...), what);
}

// launch_kernel for a kernel whose CTAs run in clusters of `cluster_x` along
// x (gridDim.x a multiple of it).
template <typename... Params, typename... Args>
int launch_kernel_cluster(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          const char* what, unsigned cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  count_launch();
  return check_cuda(cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...), what);
}

// Raise a kernel's dynamic shared-memory limit once per device (the
// attribute is per device; setting it again inside a graph capture is
// avoided).  `flags` is the caller's per-kernel bitset of configured devices.
int ensure_smem_attribute(const void* kernel, int bytes, unsigned long long* flags, const char* what);

// Encode a tiled tensor map with 16-bit elements.  `dims`/`box` are
// innermost first; `strides_bytes` has rank-1 entries (dims 1..rank-1).
// swizzle_bytes is 0, 32, 64 or 128.  Returns LDB_OK or an error code.
int encode_tiled_f16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes,
                     bool bf16 = false);

// Same for 32-bit float elements.
int encode_tiled_f32(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes);

}  // namespace ldb
