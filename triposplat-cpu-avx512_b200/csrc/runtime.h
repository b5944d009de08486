// Host-side runtime shared by the kernel families: per-thread stream, the
// host-mapped device status word, per-(device, stream) workspaces, TMA tensor
// map encoding and pointer validation.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace tsb {

// Status codes returned by every C-ABI entry point in this library.  0..-5 keep
// the meaning the reference gives them; the rest are CUDA-side conditions the
// CPU reference cannot have.
enum Status : int {
  kOk = 0,
  kNullPointer = -1,
  kBadDims = -2,
  kBadRange = -3,
  kBadAlignment = -4,
  kWorkspace = -5,
  kNotDevicePointer = -9,
  kLaunchFailed = -10,
  kDeviceFault = -11,  // a previous kernel recorded a timeout in the status word
  kNoDevice = -12,
};

cudaStream_t current_stream();

// Device pointer of this device's host-mapped status word (kernels write it).
int* device_status();
// Host view of the same word; non-zero after a kernel gave up on a wait.
int host_status();

// Workspace owned by the library, keyed by (device, stream), grown on demand
// and kept until release.  Returns nullptr if allocation fails.
void* workspace(size_t bytes, cudaStream_t stream);

// True if `p` is memory a kernel on the current device may dereference.
bool is_device_pointer(const void* p);

// Entry checks shared by all kernels: a usable device and a clean status word.
int entry_check();

// Variants that never allocate: they use this device's status word only if an earlier
// call already created it (otherwise kernels get a null status pointer and a timeout is
// reported through their exit path alone).
int entry_check_no_alloc();
int* device_status_no_alloc();

int launch_status();  // maps cudaGetLastError() to kLaunchFailed / kOk (and records the text)
void set_last_error(const char* msg);

bool encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle);

int sm_count();

// Kernel families counted / timed by LaunchScope (ids are part of the C ABI).
enum KernelId : int {
  kKGemmTc = 0,      // nf24_gemm_tc
  kKGemmSplit = 1,   // nf24_split_rows
  kKGemmSimt = 2,    // nf24_gemm_simt
  kKSdpaAttn = 3,    // sdpa_fwd_tc
  kKSdpaSplit = 4,   // sdpa_split_q + sdpa_split_kv
  kKElementwise = 5, // norms, activations, residuals, sampler updates, post-process
  kKPeerWait = 6,    // peer barrier of the multi-GPU exchanges (its time is mostly waiting)
  kKPeerCopy = 7,    // peer-memory K / V gather and partial-sum reduction
  kKNum = 8,
};

// Wrap one kernel launch: counts it and, while profiling is enabled, brackets it with
// CUDA events on `stream` (read back by triposplat_b200_profile_collect).
class LaunchScope {
 public:
  LaunchScope(int kernel_id, cudaStream_t stream);
  ~LaunchScope();
 private:
  int id_;
  cudaStream_t stream_;
  cudaEvent_t start_ = nullptr;
};

}  // namespace tsb
