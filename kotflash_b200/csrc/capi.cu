// Library-wide C-ABI pieces: version, thread-local error text, TMA descriptor
// encoding and the device-property cache.
#include <algorithm>
#include <mutex>
#include <string>

#include "kf_host.h"
#include "kf_sm100.cuh"

namespace kf {

static thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return set_error(KF_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  return KF_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

int encode_tmap_4d(CUtensorMap* map, const kf_tensor4* t, int box_inner, int box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return set_error(KF_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (t->stride[3] != 1) return set_error(KF_ERR_INVALID, "TMA view needs a contiguous last dim");
  if (!aligned16(t->ptr)) return set_error(KF_ERR_INVALID, "TMA base pointer not 16-byte aligned");
  cuuint64_t dims[4] = {(cuuint64_t)t->size[3], (cuuint64_t)t->size[2], (cuuint64_t)t->size[1],
                        (cuuint64_t)t->size[0]};
  cuuint64_t strides[3] = {(cuuint64_t)t->stride[2] * 2, (cuuint64_t)t->stride[1] * 2,
                           (cuuint64_t)t->stride[0] * 2};
  for (int i = 0; i < 3; ++i) {
    if (strides[i] % 16 != 0 || strides[i] == 0) {
      // a size-1 dimension may carry any stride; give it a legal one
      const int dim = 3 - 1 - i;  // strides[i] belongs to size[2 - i]
      if (t->size[dim] == 1) {
        strides[i] = (i == 0 ? dims[0] * 2 : strides[i - 1] * dims[i]);
        strides[i] = (strides[i] + 15) / 16 * 16;
      } else {
        return set_error(KF_ERR_INVALID, "TMA stride %llu bytes is not a multiple of 16",
                         (unsigned long long)strides[i]);
      }
    }
  }
  cuuint32_t box[4] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, t->ptr, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(KF_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return KF_OK;
}

int encode_tmap_2d_f32(CUtensorMap* map, void* ptr, int64_t rows, int64_t cols, int box_cols,
                       int box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return set_error(KF_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (!aligned16(ptr) || (cols * 4) % 16 != 0)
    return set_error(KF_ERR_INVALID, "fp32 TMA view needs 16-byte aligned base and rows");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ptr, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(KF_ERR_CUDA, "cuTensorMapEncodeTiled (fp32) failed (%d)", (int)r);
  return KF_OK;
}

DeviceGuard::DeviceGuard(const void* ptr) {
  if (!ptr) return;
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) {
    (void)cudaGetLastError();  // not a pointer the runtime knows: keep the current device
    return;
  }
  if ((attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) || attr.device < 0) return;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess) {
    (void)cudaGetLastError();
    rc_ = set_error(KF_ERR_CUDA, "cannot query the current CUDA device");
    return;
  }
  if (cur == attr.device) return;
  if (cudaSetDevice(attr.device) != cudaSuccess) {
    (void)cudaGetLastError();
    rc_ = set_error(KF_ERR_CUDA, "cannot make device %d (the tensor's) current", attr.device);
    return;
  }
  prev_ = cur;
  switched_ = true;
}

DeviceGuard::~DeviceGuard() {
  if (switched_) (void)cudaSetDevice(prev_);
}

int sm_count_current_device() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace kf

extern "C" int kf_version(void) { return 10000; }  // 1.0.0

extern "C" const char* kf_last_error(void) { return kf::g_last_error.c_str(); }

// Self-test of the bounded device wait: one thread waits on an mbarrier that
// nothing arrives on, gives up after `budget_ns`, and records the timeout in
// the status word, exactly as the attention kernels do when a peer stalls.
static __global__ void selftest_wait_kernel(int32_t* status, uint64_t budget_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    kf::mbar_init(&bar, 1);
    kf::fence_barrier_init();
    kf::mbar_wait(&bar, 0, status, budget_ns);
  }
}

extern "C" int kf_selftest_bounded_wait(int32_t* status, int64_t budget_us, void* stream) {
  if (!status || budget_us <= 0 || budget_us > 10000000)
    return kf::set_error(KF_ERR_INVALID, "kf_selftest_bounded_wait: need a status word and 0 < budget_us <= 1e7");
  kf::DeviceGuard guard(status);
  if (guard.status()) return guard.status();
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, (uint64_t)budget_us * 1000u);
  return kf::check_launch("kf_selftest_bounded_wait");
}

// Evaluates the forward kernel's packed fp32-pipe exponential on pairs of
// arguments: y[2i], y[2i+1] = exp2_poly2(x[2i], x[2i+1]).
static __global__ void selftest_exp2_kernel(const float* x, float* y, int64_t pairs) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < pairs; i += (int64_t)gridDim.x * blockDim.x) {
    float a, b;
    kf::f2_split(kf::exp2_poly2(x[2 * i], x[2 * i + 1]), a, b);
    y[2 * i] = a;
    y[2 * i + 1] = b;
  }
}

extern "C" int kf_selftest_exp2_poly(const float* x, float* y, int64_t n, void* stream) {
  if (!x || !y || n <= 0 || n % 2)
    return kf::set_error(KF_ERR_INVALID, "kf_selftest_exp2_poly: need x, y and an even n > 0");
  kf::DeviceGuard guard(x);
  if (guard.status()) return guard.status();
  const int64_t pairs = n / 2;
  const int64_t blocks = std::min<int64_t>((pairs + 255) / 256, 4096);
  selftest_exp2_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, pairs);
  return kf::check_launch("kf_selftest_exp2_poly");
}
