// common.cu — last-error storage, device status word, SM-count cache.
#include <cstdarg>
#include <atomic>
#include <mutex>
#include <vector>
#include "common.cuh"

namespace scree {

static __device__ int g_device_status = 0;

int* device_status_ptr() {
  static int* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) == cudaSuccess) cache[dev] = (int*)p;
  }
  return cache[dev];
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

int bind_device(cudaStream_t stream, const void* ptr) {
  int dev = -1;
  if (stream != nullptr && stream != cudaStreamLegacy && stream != cudaStreamPerThread) {
    SCREE_CUDA_TRY(cudaStreamGetDevice(stream, &dev));
  } else if (ptr != nullptr) {
    cudaPointerAttributes a;
    SCREE_CUDA_TRY(cudaPointerGetAttributes(&a, ptr));
    dev = a.device;
  }
  if (dev >= 0) SCREE_CUDA_TRY(cudaSetDevice(dev));
  return SCREE_OK;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

}  // namespace scree

extern "C" {

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
