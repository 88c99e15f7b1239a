// device.cu -- per-device plumbing: SM count, the device error word, the
// architecture check and TMA tensor-map encoding (through the driver entry
// point, so the library needs no link-time libcuda).
#include "common.cuh"
#include "ops.h"

#include <mutex>

namespace reef {

thread_local bool t_pdl = false;

namespace {

// One error word per device.  Bounded waits in the kernels record their
// failure code here (first error wins); read_device_error() returns and
// clears it.
__device__ int g_device_error;

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  bool init = false;
  int sms = 0;
  int major = 0, minor = 0;
  int* err = nullptr;
};

DeviceInfo g_info[kMaxDevices];
std::mutex g_mu;

DeviceInfo& info() {
  int dev = 0;
  cudaGetDevice(&dev);
  DeviceInfo& d = g_info[dev < kMaxDevices ? dev : 0];
  if (!d.init) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!d.init) {
      cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
      cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
      cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev);
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_device_error) == cudaSuccess) {
        d.err = static_cast<int*>(p);
      }
      d.init = true;
    }
  }
  return d;
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion,
                                 CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiled>(p);
    }
  });
  return fn;
}

}  // namespace

int num_sms() { return info().sms; }

int* device_error_ptr() { return info().err; }

int check_device() {
  const DeviceInfo& d = info();
  return (d.major == 10 && d.minor == 0) ? kOk : kErrUnsupported;
}

int read_device_error(int* code) {
  int* p = device_error_ptr();
  if (p == nullptr) return kErrCuda;
  int v = 0;
  if (cudaMemcpy(&v, p, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return kErrCuda;
  const int zero = 0;
  if (cudaMemcpy(p, &zero, sizeof zero, cudaMemcpyHostToDevice) != cudaSuccess)
    return kErrCuda;
  *code = v;
  return kOk;
}

namespace {
// One thread initialises an mbarrier that expects one arrival nobody makes and
// waits on it with the bounded wait: the wait must give up after `limit_ns`,
// record kDevTimeoutFull and return.
__global__ void wait_timeout_kernel(unsigned long long limit_ns, int* err, int* done) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    const bool ok = mbar_wait(&bar, 0, err, kDevTimeoutFull, limit_ns);
    *done = ok ? 1 : 2;
  }
}
}  // namespace

int selftest_wait_timeout(unsigned long long limit_ns, int* done, cudaStream_t stream) {
  if (done == nullptr || limit_ns == 0 || limit_ns > kWaitLimitNs) return kErrInvalid;
  wait_timeout_kernel<<<1, 32, 0, stream>>>(limit_ns, device_error_ptr(), done);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int make_tma_2d(CUtensorMap* map, CUtensorMapDataType type, int elem_bytes,
                const void* base, long long rows, long long cols, long long ld_elems,
                int box_cols, int box_rows, CUtensorMapSwizzle swizzle) {
  EncodeTiled fn = encode_fn();
  if (fn == nullptr) return kErrCuda;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return kErrAlignment;
  if (((ld_elems * elem_bytes) & 15) != 0) return kErrAlignment;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_elems * elem_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kErrInvalid;
}

// int8 [segs][rows][cols] with row stride ld_bytes and segment stride
// seg_bytes; boxes of box_rows x box_cols within one segment.
int make_tma_3d_i8(CUtensorMap* map, const void* base, long long rows, long long cols,
                   long long ld_bytes, long long segs, long long seg_bytes, int box_cols,
                   int box_rows) {
  EncodeTiled fn = encode_fn();
  if (fn == nullptr) return kErrCuda;
  if (segs < 1) return kErrInvalid;
  if (segs == 1) seg_bytes = ld_bytes * rows;  // unused, but must be a valid stride
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return kErrAlignment;
  if ((ld_bytes & 15) != 0 || (seg_bytes & 15) != 0) return kErrAlignment;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(segs)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld_bytes), static_cast<cuuint64_t>(seg_bytes)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kErrInvalid;
}

// [d2][d1][d0] of elem_bytes elements, dim-1 stride s1 bytes, dim-2 stride
// s2 bytes; boxes of box0 x box1 x 1.
int make_tma_3d(CUtensorMap* map, CUtensorMapDataType type, const void* base, long long d0,
                long long d1, long long d2, long long s1, long long s2, int box0, int box1,
                CUtensorMapSwizzle swizzle) {
  EncodeTiled fn = encode_fn();
  if (fn == nullptr) return kErrCuda;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return kErrAlignment;
  if ((s1 & 15) != 0 || (s2 & 15) != 0) return kErrAlignment;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1),
                        static_cast<cuuint64_t>(d2)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(s1), static_cast<cuuint64_t>(s2)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box0), static_cast<cuuint32_t>(box1), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, type, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kErrInvalid;
}

int make_tma_2d_i8(CUtensorMap* map, const void* base, long long rows, long long cols,
                   long long ld_bytes, int box_cols, int box_rows) {
  return make_tma_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base, rows, cols, ld_bytes,
                     box_cols, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace reef
