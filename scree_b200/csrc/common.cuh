// common.cuh — shared host/device helpers of libscree_b200: status codes, the
// thread-local last-error message, the device status word, dtype helpers.
#pragma once
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <type_traits>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include "../../include/scree_b200.h"

namespace scree {

// Device status word: 0 = ok, otherwise (code << 16) | site of the first error.
// It lives in common.cu; kernels receive its address (device_status_ptr()).
// (codes SCREE_DEVERR_WAIT_TIMEOUT / SCREE_DEVERR_BAD_INPUT from scree_b200.h)

__device__ __forceinline__ void record_device_error(int* status, int code, int site) {
  if (status) atomicCAS(status, 0, (code << 16) | (site & 0xFFFF));
}

// Device address of the status word on the current device (looked up once per
// device with cudaGetSymbolAddress), or nullptr if the lookup failed.
int* device_status_ptr();

// Host-side error reporting: every C entry point returns a scree_status and
// leaves a message retrievable through scree_last_error().
void set_last_error(const char* fmt, ...);

#define SCREE_CHECK_ARG(cond, ...)            \
  do {                                        \
    if (!(cond)) {                            \
      ::scree::set_last_error(__VA_ARGS__);   \
      return SCREE_ERR_INVALID;               \
    }                                         \
  } while (0)

#define SCREE_CUDA_TRY(expr)                                                        \
  do {                                                                              \
    cudaError_t _e = (expr);                                                        \
    if (_e != cudaSuccess) {                                                        \
      ::scree::set_last_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), \
                              __FILE__, __LINE__);                                  \
      return SCREE_ERR_CUDA;                                                        \
    }                                                                               \
  } while (0)

// Every kernel launch of the library goes through SCREE_LAUNCH_CHECK, which also
// counts it (scree_launch_count()).
void count_launch();
#define SCREE_LAUNCH_CHECK()            \
  do {                                  \
    SCREE_CUDA_TRY(cudaGetLastError()); \
    ::scree::count_launch();            \
  } while (0)

// Optional per-kernel timing (scree_profile_enable): CUDA events recorded on the
// launch stream around the main kernel of an entry point.
enum ProfKernel : int { PROF_ATTN_FWD = 0, PROF_ATTN_BWD = 1, PROF_NORM_FWD = 2, PROF_NORM_BWD = 3, PROF_GATHER = 4, PROF_N = 5 };
struct ProfScope {
  int kernel;
  cudaStream_t stream;
  cudaEvent_t start = nullptr;
  ProfScope(int k, cudaStream_t s);
  ~ProfScope();
};

inline size_t dtype_size(int dt) {
  switch (dt) {
    case SCREE_F16: return 2;
    case SCREE_BF16: return 2;
    case SCREE_F32: return 4;
    default: return 0;
  }
}

int num_sms();  // cached SM count of the current device

// Makes the device that owns `stream` (or, for the legacy default stream, the
// memory `ptr` points to) current on the calling thread.  Callers such as
// torch's autograd worker threads may enter with no CUDA context bound.  The
// guard puts the caller's previous device back when the entry point returns,
// if the caller had a context current (a thread with none is left bound to the
// device it used, so no context is created on a device the process never used).
struct DeviceGuard {
  int prev = -1;
  bool restore = false;
  DeviceGuard() = default;
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;
  ~DeviceGuard() {
    if (restore) cudaSetDevice(prev);
  }
};
int bind_device(cudaStream_t stream, const void* ptr, DeviceGuard* guard);
#define SCREE_BIND_DEVICE(stream, ptr)                                                   \
  ::scree::DeviceGuard _scree_device_guard;                                              \
  do {                                                                                   \
    int _rc = ::scree::bind_device((cudaStream_t)(stream), ptr, &_scree_device_guard);   \
    if (_rc != SCREE_OK) return _rc;                                                     \
  } while (0)

// Element <-> float conversion for the three activation dtypes.
template <typename T> struct Cvt;
template <> struct Cvt<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Cvt<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct Cvt<__nv_bfloat16> {
  // bf16 is the top half of an fp32: widening is a 16-bit shift (integer ALU,
  // exact), which keeps conversion-heavy loops off the special-function pipe.
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) {
    return __uint_as_float(static_cast<uint32_t>(__bfloat16_as_ushort(x)) << 16);
  }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// N floats -> N values of T; 16-bit types convert two per instruction.
template <typename T, int N>
__device__ __forceinline__ void cvt_from_f(const float* v, T* o) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value && N % 2 == 0) {
#pragma unroll
    for (int i = 0; i < N / 2; ++i)
      reinterpret_cast<__nv_bfloat162*>(o)[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  } else if constexpr (std::is_same<T, __half>::value && N % 2 == 0) {
#pragma unroll
    for (int i = 0; i < N / 2; ++i)
      reinterpret_cast<__half2*>(o)[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) o[i] = Cvt<T>::from_f(v[i]);
  }
}

// Offsets may be int32 or int64; read either as int64.
__device__ __forceinline__ int64_t load_offset(const void* offs, int is_i64, int64_t i) {
  return is_i64 ? reinterpret_cast<const int64_t*>(offs)[i]
                : static_cast<int64_t>(reinterpret_cast<const int32_t*>(offs)[i]);
}

}  // namespace scree
