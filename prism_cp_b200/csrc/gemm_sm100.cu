// Persistent tcgen05 GEMM for sm_100a:  C[M,N] (+)= rowscale[m] * sum_k A(m,k) B(n,k)
//
// Layout of the CTA (192 threads, one CTA per SM):
//   warp 0      TMA producer: 128-byte-swizzled tiles of A and B into a 4-stage ring
//   warp 1      allocates 512 TMEM columns; one elected thread issues tcgen05.mma
//               (M=128, N=256, K=16) into a double-buffered fp32 accumulator
//   warps 2..5  epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes
//               32*(w%4)..+31), scale/convert, store bf16 or fp32 (optionally +=)
// Operands may be K-major (A as [M,K], B as [N,K]) or MN-major (A as [K,M],
// B as [K,N]); MN-major tiles are loaded as 64-element-wide TMA boxes and
// described to the tensor core with LBO = box bytes, so the weight-gradient
// and input-gradient GEMMs of a linear layer run without any transpose.
// Every mbarrier wait is bounded; a timeout writes an error code to `status`
// and all roles leave their loops, release TMEM and return.
#include <cudaTypedefs.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tma_host.cuh"

namespace prism {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KiB
constexpr int B_BYTES = BN * BK * 2;  // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_THREADS = 192;
constexpr int TMEM_COLS = 512;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr int GROUP_M = 16;

struct Params {
  int M, N, K;
  void* C;
  long ldc;
  int c_fp32;
  int accumulate;
  const float* row_scale;
  int* status;
  int tiles_m, tiles_n;
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& tm, int& tn) {
  // Grouped raster: GROUP_M m-blocks share a sweep over n so that concurrently
  // running CTAs reuse both A and B tiles from L2.
  const int per_group = GROUP_M * tiles_n;
  const int g = t / per_group;
  const int first_m = g * GROUP_M;
  const int rows = min(GROUP_M, tiles_m - first_m);
  const int r = t - g * per_group;
  tm = first_m + r % rows;
  tn = r / rows;
}

template <int A_MN, int B_MN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.tiles_m * p.tiles_n;
  const int kblocks = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, p.tiles_m, p.tiles_n, tm, tn);
        const int m0 = tm * BM, n0 = tn * BN;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait_bounded(&empty[s], ph ^ 1, abort_flag, p.status, kTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          uint8_t* a_dst = smA + s * A_BYTES;
          uint8_t* b_dst = smB + s * B_BYTES;
          const int k0 = kb * BK;
          if (A_MN) {
            tma_load_2d(a_dst, &tmA, &full[s], m0, k0);
            tma_load_2d(a_dst + A_BYTES / 2, &tmA, &full[s], m0 + 64, k0);
          } else {
            tma_load_2d(a_dst, &tmA, &full[s], k0, m0);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * (B_BYTES / 4), &tmB, &full[s], n0 + 64 * j, k0);
          } else {
            tma_load_2d(b_dst, &tmB, &full[s], k0, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN, A_MN, B_MN);
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t tph = (local >> 1) & 1;
        if (!mbar_wait_bounded(&tempty[buf], tph ^ 1, abort_flag, p.status, kTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait_bounded(&full[s], ph, abort_flag, p.status, kTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smA + s * A_BYTES);
          const uint32_t b_addr = smem_u32(smB + s * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // K-major: advance 32 bytes inside the swizzled 128-byte row.
            // MN-major: advance 16 rows of 128 bytes; LBO steps between 64-wide boxes.
            const uint64_t a_desc = A_MN ? make_smem_desc_sw128(a_addr + k * 2048, A_BYTES / 2, 1024)
                                         : make_smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t b_desc = B_MN ? make_smem_desc_sw128(b_addr + k * 2048, B_BYTES / 4, 1024)
                                         : make_smem_desc_sw128(b_addr + k * 32, 16, 1024);
            umma_bf16_ss(d_tmem, a_desc, b_desc, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t tph = (local >> 1) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&tfull[buf], tph, abort_flag, p.status, kTimeoutEpilogue))) break;
      tc_fence_after();
      int tm, tn;
      tile_coords(t, p.tiles_m, p.tiles_n, tm, tn);
      const int row = tm * BM + row_in_tile;
      const float scale = (p.row_scale != nullptr && row < p.M) ? p.row_scale[row] : 1.0f;
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * BN;
#pragma unroll 1
      for (int j = 0; j < BN / 32; ++j) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + j * 32, r);
        tmem_wait_ld();
        const int col0 = tn * BN + j * 32;
        if (row >= p.M || col0 >= p.N) continue;
        const bool full_chunk = (col0 + 32 <= p.N);
        if (p.c_fp32) {
          float* out = reinterpret_cast<float*>(p.C) + (long)row * p.ldc + col0;
          if (full_chunk && ((reinterpret_cast<uintptr_t>(out) & 15) == 0)) {
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              float4 val = make_float4(__uint_as_float(r[4 * v]) * scale, __uint_as_float(r[4 * v + 1]) * scale,
                                       __uint_as_float(r[4 * v + 2]) * scale, __uint_as_float(r[4 * v + 3]) * scale);
              if (p.accumulate) {
                const float4 old = reinterpret_cast<const float4*>(out)[v];
                val.x += old.x; val.y += old.y; val.z += old.z; val.w += old.w;
              }
              reinterpret_cast<float4*>(out)[v] = val;
            }
          } else {
            for (int c = 0; c < 32 && col0 + c < p.N; ++c) {
              float val = __uint_as_float(r[c]) * scale;
              if (p.accumulate) val += out[c];
              out[c] = val;
            }
          }
        } else {
          __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.C) + (long)row * p.ldc + col0;
          if (full_chunk && ((reinterpret_cast<uintptr_t>(out) & 15) == 0)) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              float f[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(r[8 * v + e]) * scale;
              if (p.accumulate) {
                const uint4 old = reinterpret_cast<const uint4*>(out)[v];
                const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(&old);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 of = __bfloat1622float2(o2[e]);
                  f[2 * e] += of.x;
                  f[2 * e + 1] += of.y;
                }
              }
              uint4 packed = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                                        pack_bf16x2(f[6], f[7]));
              reinterpret_cast<uint4*>(out)[v] = packed;
            }
          } else {
            for (int c = 0; c < 32 && col0 + c < p.N; ++c) {
              float val = __uint_as_float(r[c]) * scale;
              if (p.accumulate) val += __bfloat162float(out[c]);
              out[c] = __float2bfloat16(val);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 2-D bf16 tensor map with 128-byte swizzle: dims {inner, outer}, row stride in elements.
CUtensorMap make_map(const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_stride_elems, uint32_t box_inner,
                     uint32_t box_outer) {
  CUtensorMap map;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) tma_encode_failed("gemm operand map", (int)r, ptr, 2, dims, strides, box);
  return map;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    C10_CUDA_CHECK(cudaGetDevice(&dev));
    C10_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

template <int A_MN, int B_MN>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(
        cudaFuncSetAttribute(gemm_kernel<A_MN, B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    configured = true;
  }
  const int tiles = p.tiles_m * p.tiles_n;
  const int grid = std::min(tiles, num_sms());
  gemm_kernel<A_MN, B_MN><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(ta, tb, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace gemm

// a: [M,K] (a_mn=false) or [K,M] (a_mn=true); b: [N,K] (b_mn=false) or [K,N] (b_mn=true).
// c: [M,N] bf16 or fp32 with unit inner stride. status: int32 device word.
void gemm_sm100(const at::Tensor& a, const at::Tensor& b, at::Tensor& c, bool a_mn, bool b_mn, bool accumulate,
                const c10::optional<at::Tensor>& row_scale, at::Tensor& status) {
  using namespace gemm;
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && c.is_cuda(), "gemm_sm100: CUDA tensors required");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm_sm100: bf16 operands");
  TORCH_CHECK(c.scalar_type() == at::kBFloat16 || c.scalar_type() == at::kFloat, "gemm_sm100: bf16/fp32 output");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && c.dim() == 2, "gemm_sm100: 2-D tensors");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && c.stride(1) == 1, "gemm_sm100: unit inner stride");
  const int64_t M = a_mn ? a.size(1) : a.size(0);
  const int64_t K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  const int64_t Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm_sm100: K mismatch ", K, " vs ", Kb);
  TORCH_CHECK(c.size(0) == M && c.size(1) == N, "gemm_sm100: output shape mismatch");
  TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0, "gemm_sm100: row strides must be multiples of 8");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(a.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(b.data_ptr()) & 15) == 0,
              "gemm_sm100: operands must be 16-byte aligned");
  TORCH_CHECK(M > 0 && N > 0 && K > 0, "gemm_sm100: empty problem");
  const c10::cuda::CUDAGuard guard(a.device());
  CUtensorMap ta = a_mn ? make_map(a.data_ptr(), M, K, a.stride(0), 64, 64)
                        : make_map(a.data_ptr(), K, M, a.stride(0), 64, BM);
  CUtensorMap tb = b_mn ? make_map(b.data_ptr(), N, K, b.stride(0), 64, 64)
                        : make_map(b.data_ptr(), K, N, b.stride(0), 64, BN);
  Params p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.C = c.data_ptr();
  p.ldc = c.stride(0);
  p.c_fp32 = c.scalar_type() == at::kFloat;
  p.accumulate = accumulate ? 1 : 0;
  p.row_scale = nullptr;
  if (row_scale.has_value()) {
    TORCH_CHECK(row_scale->scalar_type() == at::kFloat && row_scale->numel() == M, "gemm_sm100: row_scale [M] fp32");
    p.row_scale = row_scale->data_ptr<float>();
  }
  p.status = status.data_ptr<int>();
  p.tiles_m = (int)((M + BM - 1) / BM);
  p.tiles_n = (int)((N + BN - 1) / BN);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (!a_mn && !b_mn) launch<0, 0>(ta, tb, p, stream);
  else if (!a_mn && b_mn) launch<0, 1>(ta, tb, p, stream);
  else if (a_mn && !b_mn) launch<1, 0>(ta, tb, p, stream);
  else launch<1, 1>(ta, tb, p, stream);
}

}  // namespace prism
