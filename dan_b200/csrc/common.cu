// Host-side support: error text, tensor-map encoding, device queries, and the
// library-level C ABI entry points (version, last error, status word).
#include <mutex>

#include "common.cuh"

namespace dan {

static thread_local std::string g_error;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_error = buf;
}

const char* last_error() { return g_error.c_str(); }

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

int make_tmap(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int rank, const uint64_t* dims,
              const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiled fn = encode_fn();
  if (!fn) return fail(-38, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  if (reinterpret_cast<uintptr_t>(base) % 16) return fail(-22, "TMA base address %p is not 16-byte aligned", base);
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) {
      s[i] = strides_bytes[i];
      if (s[i] % 16) return fail(-22, "TMA stride %llu bytes is not a multiple of 16", (unsigned long long)s[i]);
    }
  }
  CUresult r = fn(map, dtype, rank, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(-22, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return 0;
}

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// Self-test of the bounded waits every pipelined kernel uses: one thread waits on something
// that nothing completes (kind 0: an mbarrier phase no thread arrives on; kind 1: a global
// flag no CTA sets), gives up after kWaitCycles (about a second), reports the timeout in the
// status word exactly as the production kernels do, and returns: the context stays usable.
__global__ void selftest_wait_kernel(int kind, const uint32_t* flag, int32_t* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  if (kind == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    if (!mbar_wait(&bar, 0)) report(status, kTimeoutFull);
  } else {
    if (!wait_flag(flag, 1u)) report(status, kTimeoutPartial);
  }
}

}  // namespace dan

DAN_API int dan_selftest_wait(int kind, const void* flag, int32_t* status, void* stream) {
  DAN_REQUIRE(kind == 0 || (kind == 1 && flag != nullptr), "selftest_wait: kind 0, or kind 1 with a flag word");
  dan::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      kind, static_cast<const uint32_t*>(flag), status);
  DAN_CUDA(cudaGetLastError());
  return 0;
}

DAN_API const char* dan_version(void) { return "dan_b200 0.1.0 (sm_100a)"; }

DAN_API const char* dan_last_error(void) { return dan::last_error(); }

// Reads and clears a device status word written by the kernels (0 = ok).
DAN_API int dan_read_status(int32_t* status_dev, int32_t* status_host, void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DAN_CUDA(cudaMemcpyAsync(status_host, status_dev, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  DAN_CUDA(cudaStreamSynchronize(s));
  if (*status_host != 0) DAN_CUDA(cudaMemsetAsync(status_dev, 0, sizeof(int32_t), s));
  return 0;
}
