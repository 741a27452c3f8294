// Library-wide host helpers: status strings, per-thread error messages,
// device checks and TMA descriptor encoding.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace spk {

static thread_local char t_msg[1024] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SPK_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return SPK_OK;
}

static int s_sm_count[64];
static int s_cc_major[64];
static std::mutex s_dev_mu;

static int query_device(int* dev_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(SPK_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(SPK_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(s_dev_mu);
  if (s_sm_count[dev] == 0) {
    int sms = 0, major = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    s_sm_count[dev] = sms;
    s_cc_major[dev] = major;
  }
  *dev_out = dev;
  return SPK_OK;
}

int num_sms() {
  int dev;
  if (query_device(&dev) != SPK_OK) return 148;
  return s_sm_count[dev] > 0 ? s_sm_count[dev] : 148;
}

int check_stream_device(void* /*stream*/) {
  int dev;
  int st = query_device(&dev);
  if (st != SPK_OK) return st;
  if (s_cc_major[dev] != 10)
    return fail(SPK_ERR_UNSUPPORTED, "libspk.so is built for sm_100a; device %d has compute capability %d.x",
                dev, s_cc_major[dev]);
  return SPK_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128) {
  return make_tmap_bf16_sw(map, base, rank, dims, strides_bytes, box, swizzle128 ? 128 : 0);
}

int make_tmap_bf16_sw(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes) {
  CUtensorMapSwizzle sw;
  switch (swizzle_bytes) {
    case 0: sw = CU_TENSOR_MAP_SWIZZLE_NONE; break;
    case 32: sw = CU_TENSOR_MAP_SWIZZLE_32B; break;
    case 64: sw = CU_TENSOR_MAP_SWIZZLE_64B; break;
    case 128: sw = CU_TENSOR_MAP_SWIZZLE_128B; break;
    default: return fail(SPK_ERR_INVALID, "unsupported TMA swizzle %d", swizzle_bytes);
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SPK_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (!aligned(base, 16)) return fail(SPK_ERR_ALIGN, "TMA base address must be 16-byte aligned");
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i > 0) {
      s[i - 1] = strides_bytes[i - 1];
      if (s[i - 1] % 16 != 0) return fail(SPK_ERR_ALIGN, "TMA stride %d (%llu B) not a multiple of 16", i,
                                          (unsigned long long)s[i - 1]);
    }
  }
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), d, s, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SPK_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SPK_OK;
}

// ---- self-test of the bounded wait
// One thread waits on a freshly initialised mbarrier that nothing arrives at,
// through the same mbar_wait_for loop the tensor-core pipelines use, with a
// short limit: the wait gives up, records `code` in this file's device error
// flag and the kernel returns.
__global__ void bounded_wait_probe_kernel(uint64_t limit_ns, int code) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_wait_for(&bar, 0, code, limit_ns);
  }
}

SPK_DEFINE_ERROR_READER(capi_read_device_error)

// Per-file device error readers (defined in the kernel files that spin-wait).
int gemm_read_device_error(cudaStream_t);
int gemm_il_read_device_error(cudaStream_t);
int ssa_read_device_error(cudaStream_t);
int ssa_lin_read_device_error(cudaStream_t);
int ssa_short_read_device_error(cudaStream_t);
int lif_read_device_error(cudaStream_t);
typedef int (*ErrorReader)(cudaStream_t);
static ErrorReader g_error_readers[] = {gemm_read_device_error,     gemm_il_read_device_error,
                                        ssa_read_device_error,      ssa_lin_read_device_error,
                                        ssa_short_read_device_error, lif_read_device_error,
                                        capi_read_device_error,      nullptr};

}  // namespace spk

extern "C" {

int spk_version(void) { return 1; }

const char* spk_status_string(int status) {
  switch (status) {
    case SPK_OK: return "ok";
    case SPK_ERR_INVALID: return "invalid argument";
    case SPK_ERR_SHAPE: return "unsupported shape";
    case SPK_ERR_ALIGN: return "misaligned pointer";
    case SPK_ERR_LAUNCH: return "kernel launch failed";
    case SPK_ERR_TIMEOUT: return "device wait timed out";
    case SPK_ERR_UNSUPPORTED: return "unsupported device";
    case SPK_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

const char* spk_last_error(void) { return spk::t_msg; }

int spk_device_error_check(void* stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc = SPK_OK;
  for (int i = 0; spk::g_error_readers[i]; ++i) {
    int r = spk::g_error_readers[i](st);
    if (r != SPK_OK) rc = r;
  }
  return rc;
}

int spk_test_bounded_wait(int64_t limit_ns, void* stream) {
  using namespace spk;
  SPK_REQUIRE(limit_ns > 0 && limit_ns <= 1000000000ll, SPK_ERR_INVALID, "limit %lld ns outside (0, 1 s]",
              (long long)limit_ns);
  int rc = check_stream_device(stream);
  if (rc != SPK_OK) return rc;
  bounded_wait_probe_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>((uint64_t)limit_ns, 9);
  return check_launch("bounded_wait_probe_kernel");
}

}  // extern "C"
