// Symmetric memory over NVLink/NVSwitch: one device heap per rank, mapped into
// every peer of the team through CUDA IPC, plus the P2P kernels that use it.
//
//  * symm_alloc / symm_handle / symm_open / symm_close: the heap itself. Each
//    rank cudaMalloc's its heap once, exports an IPC handle, and opens every
//    peer's handle; kernels then read and write peer memory with ordinary
//    loads and stores.
//  * Signals: a small region of each heap holds 64-bit sequence words. A writer
//    publishes with a system-scope release store to the peer's word; a reader
//    spins with acquire loads for at most a given limit and returns an error
//    status instead of hanging if the peer never arrives.
//  * p2p_gather_rows: the CP-transition reshard as one kernel - every
//    destination row block is copied straight from the owning peer's heap
//    (16-byte vector loads over NVLink) into the local layout, driven by a
//    device route table, after a bounded wait for the sender's "ready" signal;
//    it copies nothing when that wait (or any earlier one) recorded an error.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace prism {
namespace symm {

// Spin until *flag >= target; false (and an error code) after limit_ns of %globaltimer.
__device__ __forceinline__ bool wait_flag(const uint64_t* flag, uint64_t target, int* status, uint64_t limit_ns) {
  if (ld_acquire_sys(flag) >= target) return true;
  const uint64_t t0 = globaltimer();
  while (ld_acquire_sys(flag) < target) {
    if (globaltimer() - t0 > limit_ns) {
      record_error(status, kTimeoutPeer);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// Publish `value` into signal slot `slot` of every peer's heap.
__global__ void signal_all_kernel(const int64_t* peer_signal_bases, int world, int slot, uint64_t value) {
  const int r = threadIdx.x;
  if (r < world) {
    uint64_t* base = reinterpret_cast<uint64_t*>(peer_signal_bases[r]);
    st_release_sys(base + slot, value);
  }
}

// Wait until signal slots [first, first + count) of MY heap reach `value`.
__global__ void wait_all_kernel(const uint64_t* my_signals, int first, int count, uint64_t value, int* status,
                                uint64_t limit_ns) {
  const int i = threadIdx.x;
  if (i < count) wait_flag(my_signals + first + i, value, status, limit_ns);
}

// Route entry: copy `rows` rows from peer `src` (heap byte offset src_off) to
// local byte offset dst_off; rows are `row_bytes` long (multiple of 16).
struct RouteEntry {
  int64_t src_rank;
  int64_t src_off;
  int64_t dst_off;
  int64_t rows;
};

__global__ void gather_rows_kernel(const int64_t* peer_bases, int world, const RouteEntry* routes, int n_routes,
                                   const int64_t* block_route, const int64_t* block_row0, int rows_per_block,
                                   int64_t row_bytes, uint8_t* dst, int64_t dst_bytes, int* status) {
  // a bounded wait before this launch gave up (peer missing or late): copy nothing rather than rows a
  // peer may not have finished writing; the host sees the status at its next check
  if (*reinterpret_cast<volatile int*>(status) != 0) return;
  const int64_t ri = block_route[blockIdx.x];
  if (!PRISM_IN_BOUNDS(ri, n_routes, status)) return;
  const RouteEntry e = routes[ri];
  const int64_t r0 = block_row0[blockIdx.x];
  const int64_t r1 = min(e.rows, r0 + rows_per_block);
  if (!PRISM_IN_BOUNDS(e.src_rank, world, status) || !PRISM_IN_BOUNDS(r0, e.rows, status) ||
      !PRISM_IN_BOUNDS(e.dst_off + r1 * row_bytes - 1, dst_bytes, status))
    return;
  // the block's rows are contiguous on both sides: copy them as one run of 16-byte vectors, four
  // independent loads in flight per thread (NVLink reads have a long latency)
  const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(peer_bases[e.src_rank]) +
                                                    e.src_off + r0 * row_bytes);
  uint4* out = reinterpret_cast<uint4*>(dst + e.dst_off + r0 * row_bytes);
  const int64_t n = (r1 - r0) * row_bytes / 16;
  const int64_t stride = (int64_t)blockDim.x * 4;
  int64_t i = threadIdx.x;
  for (; i + 3 * blockDim.x < n; i += stride) {
    uint4 v0 = src[i], v1 = src[i + blockDim.x], v2 = src[i + 2 * blockDim.x], v3 = src[i + 3 * blockDim.x];
    out[i] = v0;
    out[i + blockDim.x] = v1;
    out[i + 2 * blockDim.x] = v2;
    out[i + 3 * blockDim.x] = v3;
  }
  for (; i < n; i += blockDim.x) out[i] = src[i];
}

}  // namespace symm

// ---------------------------------------------------------------- host API
int64_t symm_alloc(int64_t bytes) {
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, bytes));
  C10_CUDA_CHECK(cudaMemset(p, 0, bytes));
  return reinterpret_cast<int64_t>(p);
}

void symm_free(int64_t ptr) { C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

at::Tensor symm_handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  at::Tensor out = at::empty({(int64_t)sizeof(h)}, at::TensorOptions().dtype(at::kByte));
  memcpy(out.data_ptr(), &h, sizeof(h));
  return out;
}

int64_t symm_open(const at::Tensor& handle) {
  TORCH_CHECK(handle.numel() == sizeof(cudaIpcMemHandle_t), "symm_open: bad handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t ptr) { C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

// peer_signal_bases: int64 device tensor [world] of the signal-region base of every rank's heap.
void symm_signal(const at::Tensor& peer_signal_bases, int64_t slot, int64_t value) {
  const int world = peer_signal_bases.numel();
  symm::signal_all_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      peer_signal_bases.data_ptr<int64_t>(), world, (int)slot, (uint64_t)value);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// limit_ns: how long a missing peer is waited for before the error status is set (bounded, > 0).
void symm_wait(int64_t my_signal_base, int64_t first, int64_t count, int64_t value, at::Tensor& status,
               int64_t limit_ns) {
  TORCH_CHECK(count <= 32, "symm_wait: at most 32 slots");
  TORCH_CHECK(limit_ns > 0, "symm_wait: the wait needs a positive limit");
  symm::wait_all_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint64_t*>(my_signal_base), (int)first, (int)count, (uint64_t)value,
      status.data_ptr<int>(), (uint64_t)limit_ns);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// routes: int64 [n, 4] (src_rank, src_off_bytes, dst_off_bytes, rows); block tables built on host.
void symm_gather_rows(const at::Tensor& peer_bases, const at::Tensor& routes, const at::Tensor& block_route,
                      const at::Tensor& block_row0, int64_t rows_per_block, int64_t row_bytes, at::Tensor& dst,
                      at::Tensor& status) {
  TORCH_CHECK(row_bytes % 16 == 0, "symm_gather_rows: rows must be multiples of 16 bytes");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(dst.data_ptr()) & 15) == 0, "symm_gather_rows: aligned destination");
  const int blocks = block_route.numel();
  if (blocks == 0) return;
  const c10::cuda::CUDAGuard guard(dst.device());
  symm::gather_rows_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      peer_bases.data_ptr<int64_t>(), (int)peer_bases.numel(),
      reinterpret_cast<const symm::RouteEntry*>(routes.data_ptr<int64_t>()), routes.size(0),
      block_route.data_ptr<int64_t>(), block_row0.data_ptr<int64_t>(), (int)rows_per_block, row_bytes,
      reinterpret_cast<uint8_t*>(dst.data_ptr()), (int64_t)dst.nbytes(), status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace prism

namespace prism {
// A tensor view of raw device memory inside a symmetric heap (no ownership).
at::Tensor symm_tensor(int64_t ptr, std::vector<int64_t> sizes, int64_t dtype_code, int64_t device) {
  const at::ScalarType dt = static_cast<at::ScalarType>(dtype_code);
  return at::from_blob(reinterpret_cast<void*>(ptr), sizes, at::TensorOptions().dtype(dt).device(at::kCUDA, device));
}
}  // namespace prism
