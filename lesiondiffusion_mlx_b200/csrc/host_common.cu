#include "host_common.h"

#include <cstdlib>

#include <atomic>
#include <mutex>
#include <vector>

namespace ldb {

__device__ unsigned int g_device_status = 0;

namespace {
thread_local std::string t_last_error;
std::atomic<unsigned long long> g_launches{0};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}
}  // namespace

void set_last_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
}

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int check_cuda(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return LDB_OK;
  return fail(LDB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

void count_launch(int n) { g_launches.fetch_add(static_cast<unsigned long long>(n), std::memory_order_relaxed); }

int ensure_smem_attribute(const void* kernel, int bytes, unsigned long long* flags, const char* what) {
  static std::mutex mu;
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc != LDB_OK) return rc;
  std::lock_guard<std::mutex> lock(mu);
  const unsigned long long bit = 1ull << (dev & 63);
  if (*flags & bit) return LDB_OK;
  rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what);
  if (rc == LDB_OK) *flags |= bit;
  return rc;
}

unsigned int* device_status_ptr() {
  static std::mutex mu;
  static std::vector<unsigned int*> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, nullptr);
  if (!cache[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) == cudaSuccess) cache[dev] = static_cast<unsigned int*>(p);
  }
  return cache[dev];
}

namespace {
int encode_tiled(CUtensorMap* map, CUtensorMapDataType type, const void* base, int rank, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes);
}  // namespace

int encode_tiled_f16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes, bool bf16) {
  return encode_tiled(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, base, rank,
                      dims, strides_bytes, box, swizzle_bytes);
}

int encode_tiled_f32(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes) {
  return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, base, rank, dims, strides_bytes, box, swizzle_bytes);
}

namespace {
int encode_tiled(CUtensorMap* map, CUtensorMapDataType type, const void* base, int rank, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(LDB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return fail(LDB_ERR_ALIGNMENT, "tensor base address %p is not 16-byte aligned", base);
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (box[i] == 0 || box[i] > 256) return fail(LDB_ERR_SHAPE, "tensor-map box dim %d = %u", i, box[i]);
  }
  for (int i = 0; i + 1 < rank; ++i) {
    s[i] = strides_bytes[i];
    if (s[i] % 16 != 0)
      return fail(LDB_ERR_ALIGNMENT, "tensor stride %llu bytes is not a multiple of 16",
                  static_cast<unsigned long long>(s[i]));
  }
  CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
  if (swizzle_bytes == 32) sw = CU_TENSOR_MAP_SWIZZLE_32B;
  if (swizzle_bytes == 64) sw = CU_TENSOR_MAP_SWIZZLE_64B;
  if (swizzle_bytes == 128) sw = CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = fn(map, type, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LDB_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
  return LDB_OK;
}
}  // namespace

}  // namespace ldb

extern "C" {

const char* ldb_last_error(void) { return ldb::t_last_error.c_str(); }

int ldb_device_status(unsigned int* status, int reset) {
  if (!status) return ldb::fail(LDB_ERR_INVALID, "status pointer is null");
  unsigned int v = 0;
  int rc = ldb::check_cuda(cudaMemcpyFromSymbol(&v, ldb::g_device_status, sizeof(v)), "read device status");
  if (rc != LDB_OK) return rc;
  *status = v;
  if (reset) {
    unsigned int zero = 0;
    rc = ldb::check_cuda(cudaMemcpyToSymbol(ldb::g_device_status, &zero, sizeof(zero)), "reset device status");
  }
  return rc;
}

int ldb_version(void) { return LDB_ABI_VERSION; }

unsigned long long ldb_launch_count(void) { return ldb::g_launches.load(std::memory_order_relaxed); }

int ldb_clear_async(cudaStream_t stream, void* ptr, size_t bytes) {
  if (!ptr && bytes) return ldb::fail(LDB_ERR_INVALID, "clear: null pointer");
  if (!bytes) return LDB_OK;
  return ldb::check_cuda(cudaMemsetAsync(ptr, 0, bytes, stream), "clear (memset)");
}

}  // extern "C"
