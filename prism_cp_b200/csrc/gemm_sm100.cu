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
//
// AR = true turns the same kernel into the tensor-parallel GEMM -> all-reduce
// over NVLink peer memory (a row-parallel linear's output, a column-parallel
// linear's input gradient). Each of the t ranks computes its partial product
// of every tile; the tile rows are cut into t contiguous owner blocks. A rank
// visits the other owners' tiles first and its own last. For another owner's
// tile the epilogue stores the bf16 partial straight into that owner's staging
// slot (plain stores over NVLink) and publishes a per-tile sequence flag; for
// its own tile it waits (bounded) for the t-1 peer flags, adds the staged
// partials to its fp32 accumulator, writes the bf16 sum to its output and to
// every peer's output region, and publishes a per-tile result flag. After its
// tile loop each CTA copies the finished peer-owned tiles from the local output
// region into the output. The reduce-scatter half of the exchange thereby runs
// under the MMA of the following tiles; NVLink carries the same bytes as a
// reduce-scatter + all-gather. The launch is cooperative (every CTA resident),
// so a CTA never waits on a CTA of its own grid that could not be scheduled.
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

constexpr int kMaxTp = 8;

// Peer memory of one fused GEMM -> all-reduce call. Regions of rank i:
//   staging[i]   [t][R*BM][ld] bf16   slot s: partials of rank s for rank i's rows
//   outbuf[i]    [M][ld] bf16         sums of the tiles other ranks own
//   part_flag[i] [t][max_tiles] u64   slot s, tile u: rank s staged its partial
//   res_flag[i]  [max_tiles] u64      tile u: its owner wrote the sum here
struct ArParams {
  int t, me, R, max_tiles;
  long ld;
  unsigned long long seq;
  __nv_bfloat16* staging[kMaxTp];
  __nv_bfloat16* outbuf[kMaxTp];
  uint64_t* part_flag[kMaxTp];
  uint64_t* res_flag[kMaxTp];
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

__device__ __forceinline__ int ar_owner(const ArParams& ar, int tm) { return min(tm / ar.R, ar.t - 1); }

// Tile visiting order: plain grouped raster, or (AR) the owner blocks of ranks
// me+1, me+2, ..., me, each in grouped raster.
template <bool AR>
__device__ __forceinline__ void map_tile(int t, const Params& p, const ArParams& ar, int& tm, int& tn) {
  if constexpr (!AR) {
    tile_coords(t, p.tiles_m, p.tiles_n, tm, tn);
  } else {
    for (int g = 0; g < ar.t; ++g) {
      const int o = (ar.me + 1 + g) % ar.t;
      const int m_lo = o * ar.R;
      const int rows = max(0, min(m_lo + ar.R, p.tiles_m) - m_lo);
      const int n = rows * p.tiles_n;
      if (t < n) {
        tile_coords(t, rows, p.tiles_n, tm, tn);
        tm += m_lo;
        return;
      }
      t -= n;
    }
    tm = tn = 0;
  }
}

// ------------------------------------------------------------------ all-reduce epilogue
__device__ __forceinline__ void store_bf16_run(__nv_bfloat16* dst, const float* f, int ncol) {
  if (ncol == 32) {
#pragma unroll
    for (int v = 0; v < 4; ++v)
      reinterpret_cast<uint4*>(dst)[v] = make_uint4(pack_bf16x2(f[8 * v], f[8 * v + 1]), pack_bf16x2(f[8 * v + 2], f[8 * v + 3]),
                                                    pack_bf16x2(f[8 * v + 4], f[8 * v + 5]),
                                                    pack_bf16x2(f[8 * v + 6], f[8 * v + 7]));
  } else {
    for (int c = 0; c < ncol; ++c) dst[c] = __float2bfloat16(f[c]);
  }
}

__device__ __forceinline__ void add_bf16_run(float* f, const __nv_bfloat16* src, int ncol) {
  if (ncol == 32) {
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const uint4 raw = reinterpret_cast<const uint4*>(src)[v];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 x = __bfloat1622float2(h[e]);
        f[8 * v + 2 * e] += x.x;
        f[8 * v + 2 * e + 1] += x.y;
      }
    }
  } else {
    for (int c = 0; c < ncol; ++c) f[c] += __bfloat162float(src[c]);
  }
}

// One tile of the fused all-reduce, run by the 128 epilogue threads (thread =
// tile row). Returns false (jointly) when a peer wait gave up.
__device__ __forceinline__ bool ar_epilogue_tile(const Params& p, const ArParams& ar, uint32_t taddr, int tm, int tn,
                                                 int row, volatile int* abort_flag) {
  const int owner = ar_owner(ar, tm);
  const bool mine = owner == ar.me;
  const int tile_id = tm * p.tiles_n + tn;
  const long own_row0 = (long)owner * ar.R * BM;
  bool ok = true;
  if (mine) {
    bool w = true;
    for (int s = 0; s < ar.t; ++s)
      if (s != ar.me)
        w = w && wait_flag_bounded(ar.part_flag[ar.me] + (long)s * ar.max_tiles + tile_id, ar.seq, abort_flag, p.status);
    ok = named_barrier_and(w, 1, 128);
  }
  if (ok) {
    __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(p.C);
#pragma unroll 1
    for (int j = 0; j < BN / 32; ++j) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(taddr + j * 32, r);
      tmem_wait_ld();
      const int col0 = tn * BN + j * 32;
      if (row >= p.M || col0 >= p.N) continue;
      const int ncol = min(32, p.N - col0);
      float f[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) f[e] = __uint_as_float(r[e]);
      if (!mine) {
        store_bf16_run(ar.staging[owner] + ((long)ar.me * ar.R * BM + (row - own_row0)) * ar.ld + col0, f, ncol);
      } else {
        for (int s = 0; s < ar.t; ++s)
          if (s != ar.me)
            add_bf16_run(f, ar.staging[ar.me] + ((long)s * ar.R * BM + (row - own_row0)) * ar.ld + col0, ncol);
        store_bf16_run(C + (long)row * p.ldc + col0, f, ncol);
        for (int q = 0; q < ar.t; ++q)
          if (q != ar.me) store_bf16_run(ar.outbuf[q] + (long)row * ar.ld + col0, f, ncol);
      }
    }
  }
  // every thread's peer stores are ordered before the flag that publishes them
  __threadfence_system();
  ok = named_barrier_and(ok, 1, 128);
  if (ok && threadIdx.x == 64) {
    if (!mine) {
      st_release_sys(ar.part_flag[owner] + (long)ar.me * ar.max_tiles + tile_id, ar.seq);
    } else {
      for (int q = 0; q < ar.t; ++q)
        if (q != ar.me) st_release_sys(ar.res_flag[q] + tile_id, ar.seq);
    }
  }
  return ok;
}

// After the tile loop: copy the peer-owned tiles of this CTA's share (tile u =
// blockIdx.x + k * gridDim.x) from the local output region into C once their
// owners published them. Warp `quarter` copies rows 32*quarter..+31, one row
// per step, 16 bytes per lane.
__device__ __forceinline__ void ar_gather_tail(const Params& p, const ArParams& ar, int quarter, int lane,
                                               volatile int* abort_flag) {
  __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(p.C);
  const int num_tiles = p.tiles_m * p.tiles_n;
  bool ok = named_barrier_and(*abort_flag == 0, 1, 128);
  for (int u = blockIdx.x; ok && u < num_tiles; u += gridDim.x) {
    const int tm = u / p.tiles_n, tn = u % p.tiles_n;
    if (ar_owner(ar, tm) == ar.me) continue;
    ok = named_barrier_and(wait_flag_bounded(ar.res_flag[ar.me] + u, ar.seq, abort_flag, p.status), 1, 128);
    if (!ok) break;
    const int ncols = min(BN, p.N - tn * BN);
    for (int rr = 0; rr < 32; ++rr) {
      const int row = tm * BM + quarter * 32 + rr;
      if (row >= p.M) break;
      const __nv_bfloat16* src = ar.outbuf[ar.me] + (long)row * ar.ld + tn * BN;
      __nv_bfloat16* dst = C + (long)row * p.ldc + tn * BN;
      for (int c = lane * 8; c < ncols; c += 256) {
        if (c + 8 <= ncols) {
          *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(src + c);
        } else {
          for (int e = c; e < ncols; ++e) dst[e] = src[e];
        }
      }
    }
  }
}

template <int A_MN, int B_MN, bool AR>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p,
                const __grid_constant__ ArParams ar) {
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
        map_tile<AR>(t, p, ar, tm, tn);
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
      const bool got = mbar_wait_bounded(&tfull[buf], tph, abort_flag, p.status, kTimeoutEpilogue);
      // AR: every exit decision is taken jointly by the four epilogue warps, which share named barriers
      if (AR ? !named_barrier_and(got, 1, 128) : !__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      int tm, tn;
      map_tile<AR>(t, p, ar, tm, tn);
      const int row = tm * BM + row_in_tile;
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * BN;
      if constexpr (AR) {
        if (!ar_epilogue_tile(p, ar, taddr, tm, tn, row, abort_flag)) {
          tc_fence_before();
          mbar_arrive(&tempty[buf]);
          break;
        }
        tc_fence_before();
        mbar_arrive(&tempty[buf]);
        continue;
      }
      const float scale = (p.row_scale != nullptr && row < p.M) ? p.row_scale[row] : 1.0f;
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
    if constexpr (AR) ar_gather_tail(p, ar, quarter, lane, abort_flag);
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

template <int A_MN, int B_MN, bool AR>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, const ArParams& ar, cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(
        cudaFuncSetAttribute(gemm_kernel<A_MN, B_MN, AR>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    configured = true;
  }
  const int tiles = p.tiles_m * p.tiles_n;
  const int grid = std::min(tiles, num_sms());
  if constexpr (!AR) {
    gemm_kernel<A_MN, B_MN, AR><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(ta, tb, p, ar);
  } else {
    // cooperative: all CTAs are resident before any of them waits on a peer
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, gemm_kernel<A_MN, B_MN, AR>, ta, tb, p, ar));
  }
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
  const ArParams none{};
  if (!a_mn && !b_mn) launch<0, 0, false>(ta, tb, p, none, stream);
  else if (!a_mn && b_mn) launch<0, 1, false>(ta, tb, p, none, stream);
  else if (a_mn && !b_mn) launch<1, 0, false>(ta, tb, p, none, stream);
  else launch<1, 1, false>(ta, tb, p, none, stream);
}

// Tensor-parallel GEMM -> all-reduce over peer memory: c = sum over the t ranks
// of a_r b_r^T (bf16 out). regions: int64 CPU tensor [4, t] with every rank's
// staging, output-region, partial-flag and result-flag base addresses (device
// pointers valid in this process, peers' mapped through CUDA IPC); max_tiles
// is the flag capacity per slot, ld the row stride of the staging and output
// regions (>= N, multiple of 8), seq this call's sequence number (greater than
// every earlier call's on the same regions).
void gemm_allreduce_sm100(const at::Tensor& a, const at::Tensor& b, at::Tensor& c, bool a_mn, bool b_mn,
                          const at::Tensor& regions, int64_t me, int64_t max_tiles, int64_t ld, int64_t seq,
                          at::Tensor& status) {
  using namespace gemm;
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && c.is_cuda(), "gemm_allreduce: CUDA tensors required");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 && c.scalar_type() == at::kBFloat16,
              "gemm_allreduce: bf16 operands and output");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && c.dim() == 2, "gemm_allreduce: 2-D tensors");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && c.stride(1) == 1, "gemm_allreduce: unit inner stride");
  TORCH_CHECK(regions.device().is_cpu() && regions.scalar_type() == at::kLong && regions.dim() == 2 &&
                  regions.size(0) == 4 && regions.size(1) >= 2 && regions.size(1) <= kMaxTp,
              "gemm_allreduce: regions must be a CPU int64 [4, t] table, 2 <= t <= 8");
  const int64_t M = a_mn ? a.size(1) : a.size(0);
  const int64_t K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  const int64_t Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm_allreduce: K mismatch ", K, " vs ", Kb);
  TORCH_CHECK(c.size(0) == M && c.size(1) == N, "gemm_allreduce: output shape mismatch");
  TORCH_CHECK(N % 8 == 0 && c.stride(0) % 8 == 0 && ld % 8 == 0 && ld >= N, "gemm_allreduce: 16-byte rows required");
  TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0, "gemm_allreduce: row strides must be multiples of 8");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(a.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(b.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(c.data_ptr()) & 15) == 0,
              "gemm_allreduce: 16-byte aligned tensors required");
  TORCH_CHECK(M > 0 && N > 0 && K > 0, "gemm_allreduce: empty problem");
  const int t = (int)regions.size(1);
  TORCH_CHECK(me >= 0 && me < t, "gemm_allreduce: rank out of range");
  const c10::cuda::CUDAGuard guard(a.device());
  CUtensorMap ta = a_mn ? make_map(a.data_ptr(), M, K, a.stride(0), 64, 64)
                        : make_map(a.data_ptr(), K, M, a.stride(0), 64, BM);
  CUtensorMap tb = b_mn ? make_map(b.data_ptr(), N, K, b.stride(0), 64, 64)
                        : make_map(b.data_ptr(), K, N, b.stride(0), 64, BN);
  Params p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.C = c.data_ptr();
  p.ldc = c.stride(0);
  p.c_fp32 = 0;
  p.accumulate = 0;
  p.row_scale = nullptr;
  p.status = status.data_ptr<int>();
  p.tiles_m = (int)((M + BM - 1) / BM);
  p.tiles_n = (int)((N + BN - 1) / BN);
  TORCH_CHECK((int64_t)p.tiles_m * p.tiles_n <= max_tiles, "gemm_allreduce: more tiles than flag slots");
  ArParams ar{};
  ar.t = t;
  ar.me = (int)me;
  ar.R = (p.tiles_m + t - 1) / t;
  ar.max_tiles = (int)max_tiles;
  ar.ld = ld;
  ar.seq = (unsigned long long)seq;
  const int64_t* reg = regions.data_ptr<int64_t>();
  for (int i = 0; i < t; ++i) {
    ar.staging[i] = reinterpret_cast<__nv_bfloat16*>(reg[0 * t + i]);
    ar.outbuf[i] = reinterpret_cast<__nv_bfloat16*>(reg[1 * t + i]);
    ar.part_flag[i] = reinterpret_cast<uint64_t*>(reg[2 * t + i]);
    ar.res_flag[i] = reinterpret_cast<uint64_t*>(reg[3 * t + i]);
    TORCH_CHECK((reg[0 * t + i] & 15) == 0 && (reg[1 * t + i] & 15) == 0 && (reg[2 * t + i] & 7) == 0 &&
                    (reg[3 * t + i] & 7) == 0,
                "gemm_allreduce: misaligned region");
  }
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (!a_mn && !b_mn) launch<0, 0, true>(ta, tb, p, ar, stream);
  else if (!a_mn && b_mn) launch<0, 1, true>(ta, tb, p, ar, stream);
  else TORCH_CHECK(false, "gemm_allreduce: the A operand must be K-major");
}

}  // namespace prism
