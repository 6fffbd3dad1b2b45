// Cross-GPU plumbing for the peer form of the Ulysses exchange
// (vx_ulysses_pack_peers / vx_ulysses_unpack_peers): a stream-ordered flag
// barrier between ranks and CUDA IPC of the buffers the ranks exchange
// through. One process per GPU; the ranks' memories are mapped into each
// other's processes and reached over NVLink / NVSwitch by plain loads and
// stores (no NVLS objects, no TMA).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "sm100_common.cuh"
#include "vidax_cuda.h"
#include "vx_internal.h"

namespace {

constexpr int kMaxRanks = 8;
constexpr long long kDefaultTimeoutNs = 2000000000LL;  // 2 s

struct BarrierParams {
  uint32_t* flags[kMaxRanks];
  int rank, world;
  uint32_t epoch;
  long long timeout_ns;
  int* status;
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One warp; lane g < world handles rank g: announces this rank's arrival in
// rank g's array, then waits for rank g's arrival in this rank's array.
// Epochs only grow, so a rank already at a later barrier also satisfies the
// wait (the difference is compared as a signed 32-bit value).
__global__ void __launch_bounds__(32) peer_barrier_kernel(const __grid_constant__ BarrierParams p) {
  const int g = threadIdx.x;
  if (g >= p.world) return;
  __threadfence_system();  // this rank's earlier stores (and loads) before the arrival
  st_release_sys(p.flags[g] + p.rank, p.epoch);
  const uint32_t* mine = p.flags[p.rank] + g;
  const uint64_t t0 = global_ns();
  while (static_cast<int32_t>(ld_acquire_sys(mine) - p.epoch) < 0) {
    if (global_ns() - t0 > static_cast<uint64_t>(p.timeout_ns)) {
      atomicOr(p.status, vx::kDevTimeoutPeer);
      break;
    }
    __nanosleep(64);
  }
}

int fail_msg(int code, const char* msg) { return vx_internal_fail(code, msg); }

int cuda_err(cudaError_t e, const char* what) {
  char buf[256];
  snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
  return vx_internal_fail(VX_ECUDA, buf);
}

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

int address_range_fn(AddressRangeFn* fn) {
  static AddressRangeFn cached = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      cached = reinterpret_cast<AddressRangeFn>(p);
  });
  if (cached == nullptr) return fail_msg(VX_ECUDA, "cuMemGetAddressRange not available from the driver");
  *fn = cached;
  return VX_OK;
}

}  // namespace

extern "C" {

int vx_peer_barrier(const vx_peer_barrier_args* a, vx_stream_t stream) {
  if (a == nullptr) return fail_msg(VX_EINVAL, "args is NULL");
  if (a->world < 1 || a->world > kMaxRanks || a->rank < 0 || a->rank >= a->world)
    return fail_msg(VX_EINVAL, "world must be 1..8 and rank in [0, world)");
  if (a->timeout_ns < 0) return fail_msg(VX_EINVAL, "timeout_ns must be >= 0");
  BarrierParams p;
  memset(&p, 0, sizeof(p));
  for (int g = 0; g < a->world; ++g) {
    if (a->flags[g] == nullptr || (reinterpret_cast<uintptr_t>(a->flags[g]) & 3u) != 0)
      return fail_msg(VX_EINVAL, "flag arrays must be non-NULL and 4-byte aligned");
    p.flags[g] = a->flags[g];
  }
  p.rank = a->rank;
  p.world = a->world;
  p.epoch = a->epoch;
  p.timeout_ns = a->timeout_ns > 0 ? a->timeout_ns : kDefaultTimeoutNs;
  int rc = vx_internal_status_word(&p.status);
  if (rc != VX_OK) return rc;
  peer_barrier_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_err(e, "peer barrier launch");
  return VX_OK;
}

int vx_ipc_get_handle(const void* dev_ptr, char handle_out[64], int64_t* offset_out) {
  if (dev_ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
    return fail_msg(VX_EINVAL, "NULL argument");
  AddressRangeFn range;
  int rc = address_range_fn(&range);
  if (rc != VX_OK) return rc;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return fail_msg(VX_EINVAL, "dev_ptr is not device memory of this process");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_err(e, "cudaIpcGetMemHandle (memory from cudaMalloc needed)");
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  memcpy(handle_out, &h, 64);
  *offset_out = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return VX_OK;
}

int vx_ipc_open(const char handle[64], void** base_out) {
  if (handle == nullptr || base_out == nullptr) return fail_msg(VX_EINVAL, "NULL argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, 64);
  cudaError_t e = cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_err(e, "cudaIpcOpenMemHandle");
  return VX_OK;
}

int vx_ipc_close(void* base) {
  if (base == nullptr) return fail_msg(VX_EINVAL, "NULL argument");
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return cuda_err(e, "cudaIpcCloseMemHandle");
  return VX_OK;
}

}  // extern "C"
