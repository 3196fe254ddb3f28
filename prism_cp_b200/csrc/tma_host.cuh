// Host-side helpers for building TMA tensor maps (no driver library link needed:
// cuTensorMapEncodeTiled is resolved through the runtime's driver entry point).
#pragma once

#include <cstdio>
#include <stdexcept>

#include <cudaTypedefs.h>
#include <torch/extension.h>
#include <c10/cuda/CUDAException.h>

namespace prism {

// A failed encode reports every argument with C formatting and throws (pybind turns it into a
// Python RuntimeError).
[[noreturn]] inline void tma_encode_failed(const char* who, int code, const void* ptr, int rank,
                                           const cuuint64_t* dims, const cuuint64_t* strides,
                                           const cuuint32_t* box) {
  char msg[512];
  unsigned long long d[3] = {0, 0, 0}, st[2] = {0, 0};
  unsigned b[3] = {0, 0, 0};
  for (int i = 0; i < rank && i < 3; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
  }
  for (int i = 0; i + 1 < rank && i < 2; ++i) st[i] = strides[i];
  snprintf(msg, sizeof(msg),
           "%s: cuTensorMapEncodeTiled failed (code %d): ptr=%p dims=[%llu, %llu, %llu] "
           "byte strides=[%llu, %llu] box=[%u, %u, %u]",
           who, code, ptr, d[0], d[1], d[2], st[0], st[1], b[0], b[1], b[2]);
  throw std::runtime_error(msg);
}

// The encoder is a driver entry point: it needs a current context on the calling thread, which a
// fresh thread (e.g. the autograd engine's) may not have before its first runtime call.
inline void bind_current_context() {
  thread_local bool bound = false;
  if (!bound) {
    int dev = 0;
    C10_CUDA_CHECK(cudaGetDevice(&dev));
    C10_CUDA_CHECK(cudaSetDevice(dev));
    bound = true;
  }
}

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  bind_current_context();
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    C10_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && ptr != nullptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// [tokens, heads, 128] bf16 view, boxes of {64 dims, 1 head, box_rows tokens}, 128-byte swizzle.
inline CUtensorMap make_head_map(const at::Tensor& t, uint32_t box_rows) {
  TORCH_CHECK(t.dim() == 3 && t.size(2) == 128 && t.stride(2) == 1 && t.stride(1) == 128,
              "attention: tensors must be [tokens, heads, 128] with contiguous heads");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, "attention: bf16 tensors required");
  TORCH_CHECK(t.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0,
              "attention: 16-byte aligned rows required");
  CUtensorMap map;
  cuuint64_t dims[3] = {128, (cuuint64_t)t.size(1), (cuuint64_t)t.size(0)};
  cuuint64_t strides[2] = {256, (cuuint64_t)t.stride(0) * 2};
  cuuint32_t box[3] = {64, 1, box_rows};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, t.data_ptr(), dims, strides, box,
                                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) tma_encode_failed("attention head map", (int)r, t.data_ptr(), 3, dims, strides, box);
  return map;
}

inline CUtensorMap make_head_map_128(const at::Tensor& t) { return make_head_map(t, 128); }

}  // namespace prism
