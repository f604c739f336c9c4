// common.cu — last-error storage, device status word, SM-count cache.
#include <cstdarg>
#include <atomic>
#include <mutex>
#include <vector>
#include "common.cuh"
#include "sm100.cuh"

namespace scree {

static __device__ int g_device_status = 0;

// The address is looked up once per device and cached.  A cudaDeviceReset
// reloads the module at a new address; a process that resets a device must not
// use the library on it afterwards (the cached address would be stale).
int* device_status_ptr() {
  static std::atomic<int*> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  int* p = cache[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    void* a = nullptr;
    if (cudaGetSymbolAddress(&a, g_device_status) == cudaSuccess) {
      p = static_cast<int*>(a);
      cache[dev].store(p, std::memory_order_release);
    }
  }
  return p;
}

static thread_local char t_last_error[1024] = {0};

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
}

static std::atomic<long long> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// Profiling: pairs of events per kernel kind, resolved at read time.
static std::atomic<int> g_prof_on{0};
static std::mutex g_prof_mu;
static std::vector<std::pair<cudaEvent_t, cudaEvent_t>> g_prof_events[PROF_N];

ProfScope::ProfScope(int k, cudaStream_t s) : kernel(k), stream(s) {
  if (g_prof_on.load(std::memory_order_relaxed)) {
    if (cudaEventCreate(&start) == cudaSuccess) cudaEventRecord(start, stream);
    else start = nullptr;
  }
}
ProfScope::~ProfScope() {
  if (start == nullptr) return;
  cudaEvent_t stop;
  if (cudaEventCreate(&stop) != cudaSuccess) {
    cudaEventDestroy(start);
    return;
  }
  cudaEventRecord(stop, stream);
  std::lock_guard<std::mutex> g(g_prof_mu);
  g_prof_events[kernel].emplace_back(start, stop);
}

// cuCtxGetCurrent through the runtime's driver entry point (the library does
// not link libcuda directly).
using CtxGetCurrentFn = int (*)(void**);
static CtxGetCurrentFn ctx_get_current() {
  static std::atomic<CtxGetCurrentFn> fn{nullptr};
  CtxGetCurrentFn f = fn.load(std::memory_order_acquire);
  if (f == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      f = reinterpret_cast<CtxGetCurrentFn>(p);
      fn.store(f, std::memory_order_release);
    }
  }
  return f;
}

int bind_device(cudaStream_t stream, const void* ptr, DeviceGuard* guard) {
  int dev = -1;
  if (stream != nullptr && stream != cudaStreamLegacy && stream != cudaStreamPerThread) {
    SCREE_CUDA_TRY(cudaStreamGetDevice(stream, &dev));
  } else if (ptr != nullptr) {
    cudaPointerAttributes a;
    SCREE_CUDA_TRY(cudaPointerGetAttributes(&a, ptr));
    dev = a.device;
  }
  if (dev < 0) return SCREE_OK;
  int cur = -1;
  SCREE_CUDA_TRY(cudaGetDevice(&cur));
  // cudaGetDevice reports device 0 on a thread with no context bound, so
  // "cur == dev" alone does not mean the device's context is current.
  void* ctx = nullptr;
  CtxGetCurrentFn get = ctx_get_current();
  const bool has_ctx = get != nullptr && get(&ctx) == 0 && ctx != nullptr;
  if (cur == dev && has_ctx) return SCREE_OK;
  if (cur != dev && has_ctx && guard != nullptr) {
    guard->prev = cur;
    guard->restore = true;
  }
  SCREE_CUDA_TRY(cudaSetDevice(dev));
  return SCREE_OK;
}

int num_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// Self-test of the bounded waits: one thread waits on an mbarrier that nothing
// arrives on, with a limit of limit_ns.  When the wait gives up it records
// (SCREE_DEVERR_WAIT_TIMEOUT << 16) | kSiteSelfTest in the status word and the
// kernel returns normally, as every pipeline wait of the library does.
constexpr int kSiteSelfTest = 99;
__global__ void selftest_wait_kernel(int* status, unsigned long long limit_ns, int* result) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;
  abort_flag = 0;
  mbar_init(&bar, 1);
  fence_mbar_init();
  const bool ok = mbar_wait_impl(&bar, 0, &abort_flag, status, kSiteSelfTest, limit_ns);
  *result = ok ? 1 : 0;
}

}  // namespace scree

extern "C" {

int scree_selftest_wait_timeout(long long limit_ns, int* result_dev, void* stream) {
  using namespace scree;
  SCREE_CHECK_ARG(limit_ns > 0 && limit_ns <= 1000000000ll,
                  "selftest_wait_timeout: limit must be in (0, 1 s]");
  SCREE_CHECK_ARG(result_dev != nullptr, "selftest_wait_timeout: null result");
  SCREE_BIND_DEVICE(stream, result_dev);
  int* st = device_status_ptr();
  SCREE_CHECK_ARG(st != nullptr, "selftest_wait_timeout: no device status word");
  selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(st, (unsigned long long)limit_ns,
                                                          result_dev);
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}


int scree_last_error(char* buf, size_t n) {
  if (buf == nullptr || n == 0) return SCREE_ERR_INVALID;
  strncpy(buf, scree::t_last_error, n - 1);
  buf[n - 1] = 0;
  return SCREE_OK;
}

int scree_version(void) { return SCREE_ABI_VERSION; }

int scree_device_status(int* status_out, int reset) {
  if (status_out == nullptr) return SCREE_ERR_INVALID;
  int v = 0;
  SCREE_CUDA_TRY(cudaMemcpyFromSymbol(&v, scree::g_device_status, sizeof(int)));
  *status_out = v;
  if (reset) {
    int z = 0;
    SCREE_CUDA_TRY(cudaMemcpyToSymbol(scree::g_device_status, &z, sizeof(int)));
  }
  return SCREE_OK;
}

long long scree_launch_count(void) { return scree::g_launches.load(); }

int scree_profile_enable(int on) {
  scree::g_prof_on.store(on ? 1 : 0);
  return SCREE_OK;
}

int scree_profile_read(int kernel, double* total_ms, long long* launches) {
  using namespace scree;
  if (kernel < 0 || kernel >= PROF_N || !total_ms || !launches) return SCREE_ERR_INVALID;
  std::lock_guard<std::mutex> g(g_prof_mu);
  double tot = 0;
  long long n = 0;
  for (auto& pr : g_prof_events[kernel]) {
    float ms = 0.f;
    SCREE_CUDA_TRY(cudaEventSynchronize(pr.second));
    SCREE_CUDA_TRY(cudaEventElapsedTime(&ms, pr.first, pr.second));
    tot += ms;
    ++n;
    cudaEventDestroy(pr.first);
    cudaEventDestroy(pr.second);
  }
  g_prof_events[kernel].clear();
  *total_ms = tot;
  *launches = n;
  return SCREE_OK;
}

}  // extern "C"
