// Tensor-parallel reduction over NVLink peer memory (no reference counterpart).
//
// A head-sharded block ends its out / cross_out / fc2 GEMMs with one partial product per
// rank.  Instead of an all-reduce followed by a separate residual kernel, every rank reads
// the T partials straight from the ranks' device memory (CUDA IPC mappings over NVLink) and
// applies the residual update in the same pass:
//     x[i] += g[b] * (p_0[i] + p_1[i] + ... + p_{T-1}[i])      (gated residual)
//     x[i] +=         p_0[i] + ... + p_{T-1}[i]                  (residual)
// summed in rank order, so every rank computes the same bits and the replicated residual
// stream stays identical across the group.  Before the pass a one-warp barrier kernel makes
// the partials safe to read: rank r publishes a new epoch into slot r of every rank's flag
// array (release, system scope) and waits until all T slots of its own array reach it
// (acquire, system scope).  The epoch is a per-rank device counter, so a captured CUDA graph
// replays fresh epochs.  Waits are bounded (2 s wall clock) and report kDevTimeoutPeer.
// Partials are double-buffered by the caller (reduction point i writes buffer i % 2), so a
// rank can overwrite a buffer only after every rank has passed the next barrier, i.e.
// finished reading it.
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "runtime.h"

namespace tsb {
namespace peer {

constexpr int kMaxRanks = 8;

struct Ptrs {
  const float* part[kMaxRanks];
  uint32_t* flags[kMaxRanks];
};

__global__ void peer_barrier_k(Ptrs pp, int rank, int T, uint32_t* counter, int* status) {
  const int lane = threadIdx.x;
  __shared__ uint32_t epoch_s;
  if (lane == 0) {
    epoch_s = counter[0] + 1;
    counter[0] = epoch_s;
  }
  __syncwarp();
  const uint32_t epoch = epoch_s;
  if (lane < T) {
    // prior kernels' writes (the partial) are complete at this launch; order them before
    // the flag for the peers
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(pp.flags[lane] + rank), "r"(epoch)
                 : "memory");
    const uint32_t* mine = pp.flags[rank] + lane;
    const unsigned long long t0 = global_ns();
    for (uint32_t i = 0;; ++i) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if ((i & 63u) == 63u && global_ns() - t0 > kWaitBudgetNs) {
        report_error(status, kDevTimeoutPeer);
        break;
      }
      __nanosleep(64);
    }
  }
}

// x += g * sum (MODE 2) or x += sum (MODE 3), sum over the T partials in rank order
template <int MODE>
__global__ void __launch_bounds__(256) peer_reduce_residual_k(Ptrs pp, int T, float* __restrict__ x,
                                                             const float* __restrict__ gate,
                                                             int gate_ld, int64_t rows_per_batch,
                                                             int cols, int64_t n4) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 s;
    asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(s.x), "=f"(s.y), "=f"(s.z), "=f"(s.w)
                 : "l"(reinterpret_cast<const float4*>(pp.part[0]) + i));
    for (int r = 1; r < T; ++r) {
      float4 v;
      asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];"
                   : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                   : "l"(reinterpret_cast<const float4*>(pp.part[r]) + i));
      s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
    }
    float4 o = reinterpret_cast<float4*>(x)[i];
    if constexpr (MODE == 2) {
      const int64_t e = i * 4;
      const int64_t row = e / cols;
      const int c = (int)(e - row * cols);
      const float4 g = *reinterpret_cast<const float4*>(gate + (row / rows_per_batch) * gate_ld + c);
      o.x = fmaf(g.x, s.x, o.x); o.y = fmaf(g.y, s.y, o.y);
      o.z = fmaf(g.z, s.z, o.z); o.w = fmaf(g.w, s.w, o.w);
    } else {
      o.x += s.x; o.y += s.y; o.z += s.z; o.w += s.w;
    }
    reinterpret_cast<float4*>(x)[i] = o;
  }
}

static int fill_ptrs(Ptrs& pp, const uint64_t* part_ptrs, const uint64_t* flag_ptrs, int T) {
  if (T < 1 || T > kMaxRanks) return kBadDims;
  for (int r = 0; r < kMaxRanks; ++r) {
    pp.part[r] = r < T && part_ptrs ? reinterpret_cast<const float*>(part_ptrs[r]) : nullptr;
    pp.flags[r] = r < T && flag_ptrs ? reinterpret_cast<uint32_t*>(flag_ptrs[r]) : nullptr;
    if (r < T && ((part_ptrs && !part_ptrs[r]) || (flag_ptrs && !flag_ptrs[r]))) return kNullPointer;
  }
  return kOk;
}

}  // namespace peer
}  // namespace tsb

using namespace tsb;

extern "C" {

// Device buffer shareable with the other processes of one node: cudaMalloc'd, zeroed, and
// its CUDA IPC handle (64 bytes) written to handle_out.
int triposplat_b200_ipc_alloc(uint64_t bytes, void** dev_ptr, uint8_t* handle_out) {
  if (!dev_ptr || !handle_out) return kNullPointer;
  if (bytes == 0) return kBadDims;
  int st = entry_check();
  if (st != kOk) return st;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return kWorkspace;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return kLaunchFailed;
  }
  memcpy(handle_out, &h, sizeof(h));
  *dev_ptr = p;
  return kOk;
}

int triposplat_b200_ipc_free(void* dev_ptr) {
  if (!dev_ptr) return kNullPointer;
  return cudaFree(dev_ptr) == cudaSuccess ? kOk : kLaunchFailed;
}

// Map another process's buffer (its 64-byte handle) into this device's address space.
int triposplat_b200_ipc_open(const uint8_t* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return kNullPointer;
  int st = entry_check();
  if (st != kOk) return st;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return kLaunchFailed;
  }
  return kOk;
}

int triposplat_b200_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return kNullPointer;
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? kOk : kLaunchFailed;
}

// Barrier of the T ranks of a tensor-parallel group (flag_ptrs[r]: rank r's flag array of
// T uint32, as mapped in this process; counter: this rank's epoch counter, one uint32).
int triposplat_b200_peer_barrier(const uint64_t* flag_ptrs, int rank, int world, uint32_t* counter) {
  if (!flag_ptrs || !counter) return kNullPointer;
  if (rank < 0 || rank >= world) return kBadRange;
  peer::Ptrs pp;
  int st = peer::fill_ptrs(pp, nullptr, flag_ptrs, world);
  if (st != kOk) return st;
  if ((st = entry_check()) != kOk) return st;
  cudaStream_t stream = current_stream();
  {
    LaunchScope scope(kKPeerWait, stream);
    peer::peer_barrier_k<<<1, 32, 0, stream>>>(pp, rank, world, counter, device_status());
  }
  return launch_status();
}

// x[rows, cols] += gate[row / rows_per_batch] * sum_r part_r (mode 2) or += sum_r part_r
// (mode 3), part_ptrs[r] = rank r's partial as mapped here; cols % 4 == 0, 16-byte aligned.
int triposplat_b200_peer_reduce_residual_f32(const uint64_t* part_ptrs, int world, float* x,
                                             int64_t rows, int cols, int mode, const float* gate,
                                             int gate_ld, int64_t rows_per_batch) {
  if (!part_ptrs || !x) return kNullPointer;
  if (rows <= 0 || cols <= 0 || (mode != 2 && mode != 3)) return kBadDims;
  if (mode == 2 && (!gate || gate_ld < cols || rows_per_batch <= 0)) return kBadRange;
  if ((cols % 4) != 0 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (mode == 2 && ((reinterpret_cast<uintptr_t>(gate) & 15) || (gate_ld % 4))))
    return kBadAlignment;
  peer::Ptrs pp;
  int st = peer::fill_ptrs(pp, part_ptrs, nullptr, world);
  if (st != kOk) return st;
  for (int r = 0; r < world; ++r)
    if (reinterpret_cast<uintptr_t>(pp.part[r]) & 15) return kBadAlignment;
  if ((st = entry_check()) != kOk) return st;
  cudaStream_t stream = current_stream();
  const int64_t n4 = rows * (int64_t)cols / 4;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (n4 + 255) / 256;
  const unsigned grid = (unsigned)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
  {
    LaunchScope scope(kKPeerCopy, stream);
    if (mode == 2)
      peer::peer_reduce_residual_k<2><<<grid, 256, 0, stream>>>(pp, world, x, gate, gate_ld,
                                                               rows_per_batch, cols, n4);
    else
      peer::peer_reduce_residual_k<3><<<grid, 256, 0, stream>>>(pp, world, x, gate, gate_ld,
                                                               rows_per_batch, cols, n4);
  }
  return launch_status();
}

}  // extern "C"
