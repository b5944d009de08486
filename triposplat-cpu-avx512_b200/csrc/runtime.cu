// Library runtime: stream selection, device status word, workspaces, TMA maps.
#include <cudaTypedefs.h>

#include <atomic>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include <cstdio>

#include "runtime.h"

namespace tsb {

namespace {

thread_local cudaStream_t t_stream = nullptr;

struct DeviceState {
  int* host_status = nullptr;    // pinned, mapped
  int* device_status = nullptr;  // device view of host_status
  std::map<cudaStream_t, std::pair<void*, size_t>> workspaces;
  uint64_t allocations = 0;
  int sms = 0;
};

std::mutex g_mutex;
std::map<int, DeviceState> g_devices;

DeviceState* state_for_current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState& st = g_devices[dev];
  if (st.host_status == nullptr) {
    int* h = nullptr;
    if (cudaHostAlloc(reinterpret_cast<void**>(&h), sizeof(int), cudaHostAllocMapped) !=
        cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    *h = 0;
    int* d = nullptr;
    if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&d), h, 0) != cudaSuccess) {
      cudaGetLastError();
      cudaFreeHost(h);
      return nullptr;
    }
    st.host_status = h;
    st.device_status = d;
    cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return &st;
}

// Status word of the allocation-free entry points when no DeviceState exists on the
// device: one page of static host memory, page-locked and mapped (cudaHostRegister: no
// allocation) by the first such call, read by triposplat_b200_status() like host_status.
alignas(4096) int g_noalloc_status_page[1024];
std::mutex g_noalloc_status_mutex;
bool g_noalloc_status_registered = false;
int* g_noalloc_status_dev[64] = {};

int noalloc_status_value() {
  return *reinterpret_cast<volatile int*>(&g_noalloc_status_page[0]);
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

std::atomic<uint64_t> g_launches{0};
std::atomic<int> g_profiling{0};
struct TimedLaunch {
  int id;
  cudaEvent_t start, stop;
};
std::mutex g_prof_mutex;
std::vector<TimedLaunch> g_timed;

}  // namespace

// While a stream is being captured into a CUDA graph a plain event record only marks a
// dependency; cudaEventRecordExternal makes it a real record node, replayed every launch.
static void record_event(cudaEvent_t ev, cudaStream_t stream) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(ev, stream, cudaEventRecordExternal);
  else
    cudaEventRecord(ev, stream);
}

LaunchScope::LaunchScope(int kernel_id, cudaStream_t stream) : id_(kernel_id), stream_(stream) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (g_profiling.load(std::memory_order_relaxed)) {
    if (cudaEventCreate(&start_) == cudaSuccess) record_event(start_, stream_);
    else start_ = nullptr;
  }
}

LaunchScope::~LaunchScope() {
  if (start_ == nullptr) return;
  cudaEvent_t stop = nullptr;
  if (cudaEventCreate(&stop) != cudaSuccess) {
    cudaEventDestroy(start_);
    return;
  }
  record_event(stop, stream_);
  std::lock_guard<std::mutex> lock(g_prof_mutex);
  g_timed.push_back({id_, start_, stop});
}

cudaStream_t current_stream() { return t_stream; }

int* device_status() {
  DeviceState* st = state_for_current_device();
  return st ? st->device_status : nullptr;
}

int host_status() {
  DeviceState* st = state_for_current_device();
  const int s = st ? *reinterpret_cast<volatile int*>(st->host_status) : 0;
  return s != 0 ? s : noalloc_status_value();
}

int sm_count() {
  DeviceState* st = state_for_current_device();
  return st ? st->sms : 148;
}

void* workspace(size_t bytes, cudaStream_t stream) {
  DeviceState* st = state_for_current_device();
  if (!st) return nullptr;
  std::lock_guard<std::mutex> lock(g_mutex);
  auto& slot = st->workspaces[stream];
  if (slot.first != nullptr && slot.second >= bytes) return slot.first;
  // Growing: the previous buffer may still be read by work queued on `stream`.
  if (slot.first != nullptr) {
    cudaStreamSynchronize(stream);
    cudaFree(slot.first);
    slot.first = nullptr;
    slot.second = 0;
  }
  size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
  want = (want + 0xFFFFF) & ~static_cast<size_t>(0xFFFFF);
  void* p = nullptr;
  if (cudaMalloc(&p, want) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  slot.first = p;
  slot.second = want;
  st->allocations += 1;
  return p;
}

bool is_device_pointer(const void* p) {
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged ||
         (attr.type == cudaMemoryTypeHost && attr.devicePointer != nullptr);
}

int entry_check() {
  DeviceState* st = state_for_current_device();
  if (!st) return kNoDevice;
  if (*reinterpret_cast<volatile int*>(st->host_status) != 0 || noalloc_status_value() != 0)
    return kDeviceFault;
  return kOk;
}

static DeviceState* existing_state() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_mutex);
  auto it = g_devices.find(dev);
  return (it == g_devices.end() || it->second.host_status == nullptr) ? nullptr : &it->second;
}

int entry_check_no_alloc() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return kNoDevice;
  }
  DeviceState* st = existing_state();
  if (st && *reinterpret_cast<volatile int*>(st->host_status) != 0) return kDeviceFault;
  if (noalloc_status_value() != 0) return kDeviceFault;
  return kOk;
}

int* device_status_no_alloc() {
  if (DeviceState* st = existing_state()) return st->device_status;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_status_mutex);
  if (!g_noalloc_status_registered) {
    if (cudaHostRegister(g_noalloc_status_page, sizeof(g_noalloc_status_page),
                         cudaHostRegisterMapped | cudaHostRegisterPortable) != cudaSuccess) {
      cudaGetLastError();
      set_last_error("could not map the allocation-free entry's status word");
      return nullptr;
    }
    g_noalloc_status_registered = true;
  }
  if (g_noalloc_status_dev[dev] == nullptr) {
    void* d = nullptr;
    if (cudaHostGetDevicePointer(&d, g_noalloc_status_page, 0) != cudaSuccess || d == nullptr) {
      cudaGetLastError();
      set_last_error("could not map the allocation-free entry's status word");
      return nullptr;
    }
    g_noalloc_status_dev[dev] = static_cast<int*>(d);
  }
  return g_noalloc_status_dev[dev];
}

thread_local char t_last_error[256] = "";

void set_last_error(const char* msg) {
  snprintf(t_last_error, sizeof(t_last_error), "%s", msg);
}

int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return kOk;
  set_last_error(cudaGetErrorString(e));
  return kLaunchFailed;
}

bool encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  if (!g_encode) {
    set_last_error("cuTensorMapEncodeTiled unavailable");
    return false;
  }
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(map, dtype, rank, base, reinterpret_cast<const cuuint64_t*>(dims),
                        reinterpret_cast<const cuuint64_t*>(strides_bytes),
                        reinterpret_cast<const cuuint32_t*>(box), elem_strides,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "tensor map encode failed (%d): rank %u dims %llu,%llu box %u,%u dtype %d swizzle %d",
             (int)r, rank, (unsigned long long)dims[0], (unsigned long long)(rank > 1 ? dims[1] : 0),
             box[0], rank > 1 ? box[1] : 0, (int)dtype, (int)swizzle);
    set_last_error(msg);
    return false;
  }
  return true;
}

}  // namespace tsb

// ---------------------------------------------------------------------------
// C-ABI: runtime controls (no reference counterpart; the CPU library needs no
// stream and keeps its workspace thread-local)
// ---------------------------------------------------------------------------
extern "C" {

void triposplat_b200_set_stream(void* stream) {
  tsb::t_stream = reinterpret_cast<cudaStream_t>(stream);
}

void* triposplat_b200_get_stream(void) { return reinterpret_cast<void*>(tsb::t_stream); }

int triposplat_b200_status(void) { return tsb::host_status(); }

void triposplat_b200_clear_status(void) {
  tsb::DeviceState* st = tsb::state_for_current_device();
  if (st) *reinterpret_cast<volatile int*>(st->host_status) = 0;
  *reinterpret_cast<volatile int*>(&tsb::g_noalloc_status_page[0]) = 0;
}

int triposplat_b200_workspace_reserve(uint64_t bytes) {
  return tsb::workspace(bytes, tsb::t_stream) ? 0 : tsb::kWorkspace;
}

int triposplat_b200_workspace_stats(uint64_t* allocations, uint64_t* capacity_bytes) {
  if (!allocations || !capacity_bytes) return tsb::kNullPointer;
  tsb::DeviceState* st = tsb::state_for_current_device();
  if (!st) return tsb::kNoDevice;
  std::lock_guard<std::mutex> lock(tsb::g_mutex);
  uint64_t cap = 0;
  for (auto& kv : st->workspaces) cap += kv.second.second;
  *allocations = st->allocations;
  *capacity_bytes = cap;
  return 0;
}

void triposplat_b200_workspace_release(void) {
  tsb::DeviceState* st = tsb::state_for_current_device();
  if (!st) return;
  cudaDeviceSynchronize();
  std::lock_guard<std::mutex> lock(tsb::g_mutex);
  for (auto& kv : st->workspaces)
    if (kv.second.first) cudaFree(kv.second.first);
  st->workspaces.clear();
}

int triposplat_b200_abi_version(void) { return 1; }

// Text of the last CUDA / tensor-map error seen by this thread's calls ("" if none).
const char* triposplat_b200_last_error(void) { return tsb::t_last_error; }

uint64_t triposplat_b200_launch_count(void) {
  return tsb::g_launches.load(std::memory_order_relaxed);
}

void triposplat_b200_profile_enable(int on) { tsb::g_profiling.store(on ? 1 : 0); }

// Waits for every bracketed launch recorded so far, then returns per kernel family
// (index = KernelId, n entries) the launch count and the summed device time in ms,
// and forgets them.
// With keep != 0 the events stay registered (e.g. because a captured CUDA graph still
// records into them on every replay); each read then reflects their latest recording.
int triposplat_b200_profile_collect2(uint64_t* launches, double* total_ms, int n, int keep) {
  if (!launches || !total_ms || n <= 0) return tsb::kNullPointer;
  for (int i = 0; i < n; ++i) { launches[i] = 0; total_ms[i] = 0.0; }
  std::vector<tsb::TimedLaunch> items;
  {
    std::lock_guard<std::mutex> lock(tsb::g_prof_mutex);
    if (keep) items = tsb::g_timed;
    else items.swap(tsb::g_timed);
  }
  int st = 0;
  for (auto& it : items) {
    float ms = 0.0f;
    if (cudaEventSynchronize(it.stop) == cudaSuccess &&
        cudaEventElapsedTime(&ms, it.start, it.stop) == cudaSuccess) {
      if (it.id >= 0 && it.id < n) { launches[it.id] += 1; total_ms[it.id] += ms; }
    } else {
      tsb::set_last_error(cudaGetErrorString(cudaGetLastError()));
      st = tsb::kLaunchFailed;
    }
    if (!keep) {
      cudaEventDestroy(it.start);
      cudaEventDestroy(it.stop);
    }
  }
  return st;
}

int triposplat_b200_profile_collect(uint64_t* launches, double* total_ms, int n) {
  return triposplat_b200_profile_collect2(launches, total_ms, n, 0);
}

}  // extern "C"
