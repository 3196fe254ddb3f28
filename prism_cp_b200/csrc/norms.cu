// Row-normalisation kernels (one warp per row, 16-byte vector accesses).
//
// One kernel family covers the three norms of the hybrid decoder:
//   RMSNorm          y = x * rsqrt(mean(x^2) + eps) * w
//   gated RMSNorm    y = x * rsqrt(mean(x^2) + eps) * w * silu(z)   (GDN output norm, per head)
//   L2 norm          y = x * rsqrt(sum(x^2) + eps)                 (GDN q/k, per head)
// `inv_n` selects mean (1/n) or sum (1) of squares. The forward stores the fp32
// reciprocal norm per row for the backward. Weight gradients are reduced in two
// stages: per-block partial sums in shared memory, then a column-sum kernel.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace prism {
namespace {

constexpr int kWarpsPerBlock = 8;

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 v = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                       pack_bf16x2(f[6], f[7]));
  *reinterpret_cast<uint4*>(p) = v;
}

// Rows are addressed as row -> (row / heads, row % heads): element (r, i) of the
// logical [rows, n] matrix lives at base + (r / heads) * stride + (r % heads) * n + i.
template <bool HAS_W, bool GATED>
__global__ void rownorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, long x_stride,
                                   const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ z,
                                   long z_stride, __nv_bfloat16* __restrict__ y, long y_stride,
                                   float* __restrict__ rstd, int rows, int heads, int n, float inv_n, float eps) {
  const int warp = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const long tok = warp / heads, hd = warp % heads;
  const __nv_bfloat16* xr = x + tok * x_stride + hd * n;
  float ss = 0.f;
  for (int i = lane * 8; i < n; i += 256) {
    float f[8];
    load8(xr + i, f);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss * inv_n + eps);
  if (lane == 0) rstd[warp] = r;
  __nv_bfloat16* yr = y + tok * y_stride + hd * n;
  const __nv_bfloat16* zr = GATED ? z + tok * z_stride + hd * n : nullptr;
  for (int i = lane * 8; i < n; i += 256) {
    float f[8], wf[8], zf[8];
    load8(xr + i, f);
    if (HAS_W) load8(w + i, wf);
    if (GATED) load8(zr + i, zf);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float v = f[e] * r;
      if (HAS_W) v *= wf[e];
      if (GATED) v *= silu(zf[e]);
      f[e] = v;
    }
    store8(yr + i, f);
  }
}

// Weight-gradient accumulators a lane keeps in registers (8 columns per 256-column chunk): rows
// of up to kRegChunks * 256 elements sum their dw terms there and reach shared memory once per
// warp instead of once per row; wider rows add each term to shared memory directly.
constexpr int kRegChunks = 8;

template <bool HAS_W, bool GATED>
__device__ __forceinline__ void rownorm_bwd_chunk(const __nv_bfloat16* xr, const __nv_bfloat16* dyr,
                                                  const __nv_bfloat16* w, const __nv_bfloat16* zr,
                                                  __nv_bfloat16* dxr, __nv_bfloat16* dzr, int i, float r, float c,
                                                  float* dwv) {
  float xf[8], dyf[8], wf[8], zf[8], out[8], dzo[8];
  load8(xr + i, xf);
  load8(dyr + i, dyf);
  if (HAS_W) load8(w + i, wf);
  if (GATED) load8(zr + i, zf);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float wv = HAS_W ? wf[e] : 1.f;
    float gate = 1.f;
    if (GATED) {
      const float s = sigmoidf_(zf[e]);
      gate = zf[e] * s;
      const float dsilu = s * (1.f + zf[e] * (1.f - s));
      dzo[e] = dyf[e] * xf[e] * r * wv * dsilu;
    }
    const float g = dyf[e] * wv * gate;
    out[e] = g * r - xf[e] * c;
    if (HAS_W) dwv[e] = dyf[e] * gate * xf[e] * r;
  }
  store8(dxr + i, out);
  if (GATED) store8(dzr + i, dzo);
}

template <bool HAS_W, bool GATED>
__global__ void rownorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, long dy_stride,
                                   const __nv_bfloat16* __restrict__ x, long x_stride,
                                   const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ z,
                                   long z_stride, const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx,
                                   long dx_stride, __nv_bfloat16* __restrict__ dz, long dz_stride,
                                   float* __restrict__ dw_partial, int rows, int heads, int n, float inv_n) {
  extern __shared__ float dw_s[];
  if (HAS_W) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) dw_s[i] = 0.f;
    __syncthreads();
  }
  const int lane = threadIdx.x & 31;
  const int warps_total = gridDim.x * kWarpsPerBlock;
  const bool reg_acc = HAS_W && n <= kRegChunks * 256;
  float acc[kRegChunks][8];
#pragma unroll
  for (int k = 0; k < kRegChunks; ++k)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[k][e] = 0.f;
  for (int row = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows; row += warps_total) {
    const long tok = row / heads, hd = row % heads;
    const __nv_bfloat16* xr = x + tok * x_stride + hd * n;
    const __nv_bfloat16* dyr = dy + tok * dy_stride + hd * n;
    const __nv_bfloat16* zr = GATED ? z + tok * z_stride + hd * n : nullptr;
    const float r = rstd[row];
    // g = dy * w * gate;   dot = sum g * x
    float dot = 0.f;
    for (int i = lane * 8; i < n; i += 256) {
      float xf[8], gf[8], wf[8], zf[8];
      load8(xr + i, xf);
      load8(dyr + i, gf);
      if (HAS_W) load8(w + i, wf);
      if (GATED) load8(zr + i, zf);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float g = gf[e];
        if (HAS_W) g *= wf[e];
        if (GATED) g *= silu(zf[e]);
        dot += g * xf[e];
      }
    }
    dot = warp_sum(dot);
    const float c = dot * r * r * r * inv_n;
    __nv_bfloat16* dxr = dx + tok * dx_stride + hd * n;
    __nv_bfloat16* dzr = GATED ? dz + tok * dz_stride + hd * n : nullptr;
    if (reg_acc) {
#pragma unroll
      for (int k = 0; k < kRegChunks; ++k) {
        const int i = lane * 8 + k * 256;
        if (i < n) {
          float dwv[8];
          rownorm_bwd_chunk<HAS_W, GATED>(xr, dyr, w, zr, dxr, dzr, i, r, c, dwv);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[k][e] += dwv[e];
        }
      }
    } else {
      for (int i = lane * 8; i < n; i += 256) {
        float dwv[8];
        rownorm_bwd_chunk<HAS_W, GATED>(xr, dyr, w, zr, dxr, dzr, i, r, c, dwv);
        if (HAS_W) {
#pragma unroll
          for (int e = 0; e < 8; ++e) atomicAdd(&dw_s[i + e], dwv[e]);
        }
      }
    }
  }
  if (HAS_W) {
    if (reg_acc) {
#pragma unroll
      for (int k = 0; k < kRegChunks; ++k) {
        const int i = lane * 8 + k * 256;
        if (i < n) {
#pragma unroll
          for (int e = 0; e < 8; ++e) atomicAdd(&dw_s[i + e], acc[k][e]);
        }
      }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) dw_partial[(long)blockIdx.x * n + i] = dw_s[i];
  }
}

__global__ void column_sum_kernel(const float* __restrict__ partial, int parts, int n, float* __restrict__ out_f32,
                                  __nv_bfloat16* __restrict__ out_bf16) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float s = 0.f;
  for (int p = 0; p < parts; ++p) s += partial[(long)p * n + i];
  if (out_f32 != nullptr) out_f32[i] = s;
  if (out_bf16 != nullptr) out_bf16[i] = __float2bfloat16(s);
}

void check_rows(const at::Tensor& t, const char* name, int n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, name, ": CUDA bf16 tensor required");
  TORCH_CHECK(t.stride(-1) == 1, name, ": unit inner stride required");
  TORCH_CHECK(n % 8 == 0, name, ": normalised length must be a multiple of 8");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, name, ": 16-byte alignment required");
  TORCH_CHECK(t.dim() < 2 || (t.stride(0) % 8) == 0, name, ": row stride must be a multiple of 8 elements");
}

}  // namespace

// x: [T, heads*n] (row stride may exceed heads*n). Returns nothing; writes y and rstd [T*heads].
void rownorm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& z,
                 at::Tensor& y, at::Tensor& rstd, int64_t heads, int64_t n, double inv_n, double eps) {
  check_rows(x, "rownorm_fwd.x", n);
  check_rows(y, "rownorm_fwd.y", n);
  const c10::cuda::CUDAGuard guard(x.device());
  const int rows = (int)(x.size(0) * heads);
  const int blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  auto stream = at::cuda::getCurrentCUDAStream();
  const __nv_bfloat16* wp = w ? reinterpret_cast<const __nv_bfloat16*>(w->data_ptr()) : nullptr;
  const __nv_bfloat16* zp = z ? reinterpret_cast<const __nv_bfloat16*>(z->data_ptr()) : nullptr;
  const long zs = z ? z->stride(0) : 0;
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  if (z) check_rows(*z, "rownorm_fwd.z", n);
#define PRISM_NORM_FWD(HW, G)                                                                                      \
  rownorm_fwd_kernel<HW, G><<<blocks, kWarpsPerBlock * 32, 0, stream>>>(xp, x.stride(0), wp, zp, zs, yp,          \
                                                                      y.stride(0), rstd.data_ptr<float>(), rows,  \
                                                                      (int)heads, (int)n, (float)inv_n, (float)eps)
  if (wp && zp) PRISM_NORM_FWD(true, true);
  else if (wp) PRISM_NORM_FWD(true, false);
  else if (zp) PRISM_NORM_FWD(false, true);
  else PRISM_NORM_FWD(false, false);
#undef PRISM_NORM_FWD
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Returns dw (fp32 [n]) when w is given; writes dx and (gated) dz.
c10::optional<at::Tensor> rownorm_bwd(const at::Tensor& dy, const at::Tensor& x, const c10::optional<at::Tensor>& w,
                                      const c10::optional<at::Tensor>& z, const at::Tensor& rstd, at::Tensor& dx,
                                      const c10::optional<at::Tensor>& dz, int64_t heads, int64_t n, double inv_n) {
  check_rows(dy, "rownorm_bwd.dy", n);
  check_rows(x, "rownorm_bwd.x", n);
  check_rows(dx, "rownorm_bwd.dx", n);
  const c10::cuda::CUDAGuard guard(x.device());
  const int rows = (int)(x.size(0) * heads);
  int sms = 0;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, x.get_device()));
  const int blocks = std::max(1, std::min((rows + kWarpsPerBlock - 1) / kWarpsPerBlock, sms * 4));
  auto stream = at::cuda::getCurrentCUDAStream();
  const bool has_w = w.has_value(), gated = z.has_value();
  at::Tensor partial;
  if (has_w) partial = at::empty({blocks, n}, x.options().dtype(at::kFloat));
  const __nv_bfloat16* wp = has_w ? reinterpret_cast<const __nv_bfloat16*>(w->data_ptr()) : nullptr;
  const __nv_bfloat16* zp = gated ? reinterpret_cast<const __nv_bfloat16*>(z->data_ptr()) : nullptr;
  __nv_bfloat16* dzp = gated ? reinterpret_cast<__nv_bfloat16*>(dz->data_ptr()) : nullptr;
  const long zs = gated ? z->stride(0) : 0, dzs = gated ? dz->stride(0) : 0;
  const size_t smem = has_w ? n * sizeof(float) : 0;
  auto dyp = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto dxp = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  float* pp = has_w ? partial.data_ptr<float>() : nullptr;
#define PRISM_NORM_BWD(HW, G)                                                                                  \
  rownorm_bwd_kernel<HW, G><<<blocks, kWarpsPerBlock * 32, smem, stream>>>(                                  \
      dyp, dy.stride(0), xp, x.stride(0), wp, zp, zs, rstd.data_ptr<float>(), dxp, dx.stride(0), dzp, dzs, pp, \
      rows, (int)heads, (int)n, (float)inv_n)
  if (has_w && gated) PRISM_NORM_BWD(true, true);
  else if (has_w) PRISM_NORM_BWD(true, false);
  else if (gated) PRISM_NORM_BWD(false, true);
  else PRISM_NORM_BWD(false, false);
#undef PRISM_NORM_BWD
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (!has_w) return c10::nullopt;
  at::Tensor dw = at::empty({n}, x.options().dtype(at::kFloat));
  column_sum_kernel<<<(n + 255) / 256, 256, 0, stream>>>(partial.data_ptr<float>(), blocks, (int)n,
                                                          dw.data_ptr<float>(), nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dw;
}

}  // namespace prism

// ============================================================================
// Allocation-free RMSNorm backward (C ABI), declared with its full contract in
// prism_noalloc.h. This entry point has no counterpart in the reference
// framework: it serves callers that cannot allocate device memory (no caching
// allocator, allocation forbidden while a step is in flight, or a fixed memory
// budget). Its only working memory, the per-block partial sums of dW, lives in
// the fixed array below instead of a fresh allocation.
// ============================================================================
#include <mutex>

#include "prism_noalloc.h"

namespace prism {
namespace {

constexpr int kNoAllocScratchFloats = PRISM_NOALLOC_SCRATCH_BYTES / sizeof(float);  // 4 MiB of fp32 sums
constexpr int kNoAllocMaxN = PRISM_NOALLOC_MAX_N;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

std::mutex g_noalloc_mutex;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {};
int g_noalloc_sms[kNoAllocMaxDevices] = {};

bool aligned_to(const void* p, uintptr_t bytes) { return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0; }

// Device address of the scratch array on the current device (looked up once).
int noalloc_setup(int device, float** out, int* sms) {
  std::lock_guard<std::mutex> guard(g_noalloc_mutex);
  if (g_noalloc_ptr[device] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) {
      return PRISM_NOALLOC_SETUP_FAILED;
    }
    int count = 0;
    if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
      return PRISM_NOALLOC_SETUP_FAILED;
    }
    g_noalloc_ptr[device] = static_cast<float*>(ptr);
    g_noalloc_sms[device] = count;
  }
  *out = g_noalloc_ptr[device];
  *sms = g_noalloc_sms[device];
  return PRISM_NOALLOC_OK;
}

}  // namespace
}  // namespace prism

extern "C" __attribute__((visibility("default"))) const char* prism_noalloc_error_string(int code) {
  switch (code) {
    case PRISM_NOALLOC_OK: return "ok";
    case PRISM_NOALLOC_BAD_ARGUMENT:
      return "bad argument (null or misaligned pointer, rows < 1, or n not a multiple of 8)";
    case PRISM_NOALLOC_TOO_LARGE: return "n exceeds the 8192 maximum of the fixed scratch array";
    case PRISM_NOALLOC_SETUP_FAILED: return "could not resolve the scratch array on the current device";
    case PRISM_NOALLOC_LAUNCH_FAILED: return "kernel launch failed";
    case PRISM_NOALLOC_PENDING_ERROR: return "a CUDA error from earlier work was pending; nothing was launched";
    default: return "unknown error";
  }
}

// dx = d/dx and dw = d/dw of y = x * rsqrt(mean(x^2) + eps) * w, given dy and the
// forward's reciprocal norms, on `stream`, without allocating device memory.
extern "C" __attribute__((visibility("default"))) int prism_rmsnorm_bwd_noalloc(
    const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw, int rows, int n,
    cudaStream_t stream) {
  using namespace prism;
  if (dy == nullptr || x == nullptr || w == nullptr || rstd == nullptr || dx == nullptr || dw == nullptr ||
      rows < 1 || n < 8 || n % 8 != 0) {
    return PRISM_NOALLOC_BAD_ARGUMENT;
  }
  if (!aligned_to(dy, 16) || !aligned_to(x, 16) || !aligned_to(w, 16) || !aligned_to(dx, 16) ||
      !aligned_to(rstd, 4) || !aligned_to(dw, 4)) {
    return PRISM_NOALLOC_BAD_ARGUMENT;
  }
  if (n > kNoAllocMaxN) return PRISM_NOALLOC_TOO_LARGE;
  // an error left by the caller's earlier work is reported as such, not as this call's launch failure
  if (cudaPeekAtLastError() != cudaSuccess) return PRISM_NOALLOC_PENDING_ERROR;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kNoAllocMaxDevices) {
    return PRISM_NOALLOC_SETUP_FAILED;
  }
  float* scratch = nullptr;
  int sms = 0;
  const int setup = noalloc_setup(device, &scratch, &sms);
  if (setup != PRISM_NOALLOC_OK) return setup;
  int blocks = std::min((rows + kWarpsPerBlock - 1) / kWarpsPerBlock, sms * 4);
  blocks = std::max(1, std::min(blocks, kNoAllocScratchFloats / n));
  const auto* dyp = static_cast<const __nv_bfloat16*>(dy);
  const auto* xp = static_cast<const __nv_bfloat16*>(x);
  const auto* wp = static_cast<const __nv_bfloat16*>(w);
  auto* dxp = static_cast<__nv_bfloat16*>(dx);
  rownorm_bwd_kernel<true, false><<<blocks, kWarpsPerBlock * 32, n * sizeof(float), stream>>>(
      dyp, n, xp, n, wp, nullptr, 0, rstd, dxp, n, nullptr, 0, scratch, rows, 1, n, 1.0f / n);
  if (cudaGetLastError() != cudaSuccess) return PRISM_NOALLOC_LAUNCH_FAILED;
  column_sum_kernel<<<(n + 255) / 256, 256, 0, stream>>>(scratch, blocks, n, dw, nullptr);
  if (cudaGetLastError() != cudaSuccess) return PRISM_NOALLOC_LAUNCH_FAILED;
  return PRISM_NOALLOC_OK;
}
