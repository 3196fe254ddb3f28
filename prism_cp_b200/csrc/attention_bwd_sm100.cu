// Flash-attention backward on tcgen05 (sm_100a), varlen / causal / GQA, head_dim 128.
//
// Two atomic-free kernels share the CTA shape of the forward (warps 0-7 compute, warps w
// and w + 4 on TMEM lanes 32(w % 4).. == tile rows, each taking half of the columns; warp 8
// TMA producer, warp 9 MMA issuer):
//   kv kernel  one CTA per (128-key tile, kv head), looping over the query heads
//              of the GQA group and the query tiles that see the keys:
//                S^T = K Q^T, dP^T = V dO^T            (TMEM cols 0-255)
//                P^T = exp2(S^T*c - lse), dS^T = P^T (dP^T - D)  -> smem (bf16)
//                dV += P^T dO, dK += dS^T Q            (TMEM cols 256-511)
//   q kernel   one CTA per (128-query tile, query head), looping over key tiles:
//                S = Q K^T, dP = dO V^T, dS = P (dP - D) -> smem, dQ += dS K
// dK/dV/dQ are written once in bf16; nothing is accumulated with atomics, so the
// result is deterministic. D = rowsum(dO * O) comes from a small preprocess kernel.
// For context-parallel ring steps the caller passes the merged (global) O and LSE,
// which makes P the correctly normalised global probabilities for that KV chunk.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tma_host.cuh"
#include "attention_peer.cuh"

#include <type_traits>

namespace prism {
namespace attnb {

constexpr int D = 128;
constexpr int TILE = 128;
constexpr int TILE_BYTES = 128 * D * 2;  // 32 KiB
constexpr int HALF = TILE_BYTES / 2;     // one 64-column box
constexpr float kLog2e = 1.4426950408889634f;

struct Params {
  const int* cu_q;
  const int* cu_k;
  const int* tiles;
  int hq, hkv;
  int causal;
  float scale;       // softmax scale
  const float* lse;  // [hq, Tq] natural log
  const float* dsum; // [hq, Tq]
  int tq;
  int tk;            // rows of K / V / dK / dV (bounds of the debug build)
  __nv_bfloat16* out;  // dK / dV (kv kernel) or dQ (q kernel)
  __nv_bfloat16* out2;
  long out_stride;
  int* status;
};

__device__ __forceinline__ void write_chunk_sw128(uint8_t* base, int row, int chunk, uint4 val) {
  const int blk = chunk >> 3, cc = chunk & 7;
  *reinterpret_cast<uint4*>(base + blk * HALF + row * 128 + ((cc ^ (row & 7)) << 4)) = val;
}

__device__ __forceinline__ void named_sync_compute() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ void named_sync_kv() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// K-major operand (rows x 128 dims as two 64-dim boxes); k = 16-element step.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t base, int k) {
  return make_smem_desc_sw128(base + (k >> 2) * HALF + (k & 3) * 32, 16, 1024);
}
// MN-major operand: rows are the reduction dim, two 64-wide boxes along MN.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t base, int k) {
  return make_smem_desc_sw128(base + k * 2048, HALF, 1024);
}

// ------------------------------------------------------------------ dK, dV
// One CTA per (128-key tile, kv head). Query tiles of 64 rows stream through a
// two-stage TMA ring; S^T / dP^T for the next query tile are computed into the
// other half of a double-buffered TMEM region while the compute warps turn the
// current one into P^T and dS^T, so TMA, tensor cores and the softmax-gradient
// math overlap.
//   TMEM: S^T [0,64) / [64,128), dP^T [128,192) / [192,256), dV [256,384), dK [384,512)
// Src = PeerTiles: this rank's keys of a zigzag team; tiles hold (seq, global
// position of the first key, its local row); Q / dO tiles and their LSE / D rows
// are read from the rank that owns each query tile.
// The dK/dV kernel runs eight compute warps: warps w and w + 4 share TMEM lanes (key rows) 32(w % 4)..
// and split the 64 query columns of each iteration, so every SM sub-partition has two warps of
// P^T / dS^T math to interleave (the math, not the tensor cores, bounds an iteration). Warp 8 is the
// TMA producer, warp 9 issues the MMAs.
constexpr int KV_THREADS = 320;
constexpr int KV_COMPUTE = 256;
constexpr int KV_QT = 64;                    // query rows per iteration
constexpr int KV_STAGES = 3;                 // Q / dO ring: the load of tile it + 2 overlaps the dK/dV MMAs of it
constexpr int KV_QBYTES = KV_QT * D * 2;     // 16 KiB: 64 rows x 128 dims (two 64-dim boxes)
constexpr int KV_QHALF = KV_QBYTES / 2;
constexpr int KV_PBYTES = 128 * KV_QT * 2;   // 16 KiB: 128 keys x 64 queries
constexpr int KV_OFF_Q = 2 * TILE_BYTES;                         // Q[KV_STAGES]
constexpr int KV_OFF_DO = KV_OFF_Q + KV_STAGES * KV_QBYTES;      // dO[KV_STAGES]
constexpr int KV_OFF_PT = KV_OFF_DO + KV_STAGES * KV_QBYTES;
constexpr int KV_OFF_DST = KV_OFF_PT + KV_PBYTES;
constexpr int KV_OFF_STAT = KV_OFF_DST + KV_PBYTES;      // lse[2][64], dsum[2][64]
constexpr int KV_OFF_BAR = KV_OFF_STAT + 4 * KV_QT * 4;

template <class Src>
__global__ void __launch_bounds__(KV_THREADS, 1)
    attn_bwd_kv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                       Params p, const __grid_constant__ Src src) {
  constexpr bool PEER = std::is_same<Src, PeerTiles>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + TILE_BYTES;
  uint8_t* sPT = smem + KV_OFF_PT;
  uint8_t* sdST = smem + KV_OFF_DST;
  float* lse_s = reinterpret_cast<float*>(smem + KV_OFF_STAT);   // [2][64]
  float* dsum_s = lse_s + 2 * KV_QT;                             // [2][64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + KV_OFF_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;                  // [KV_STAGES]
  uint64_t* q_empty = bars + 1 + KV_STAGES;     // [KV_STAGES]
  uint64_t* s_full = bars + 1 + 2 * KV_STAGES;  // [2]
  uint64_t* s_free = s_full + 2;                // [2]
  uint64_t* p_full = s_full + 4;
  uint64_t* mma_done = s_full + 5;
  uint64_t* acc_done = s_full + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(s_full + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kv_head = blockIdx.y;
  const int rep = p.hq / p.hkv;
  int seq, k0, q_seg, q_len, k_seg, k_len;
  if constexpr (PEER) {
    seq = p.tiles[3 * blockIdx.x];
    k0 = p.tiles[3 * blockIdx.x + 1];
    k_seg = p.tiles[3 * blockIdx.x + 2] - k0;
    q_len = k_len = src.seq_n[seq];
    q_seg = 0;
  } else {
    seq = p.tiles[2 * blockIdx.x];
    k0 = p.tiles[2 * blockIdx.x + 1] * TILE;
    q_seg = p.cu_q[seq];
    q_len = p.cu_q[seq + 1] - q_seg;
    k_seg = p.cu_k[seq];
    k_len = p.cu_k[seq + 1] - k_seg;
  }
  const int n_qt = (q_len + KV_QT - 1) / KV_QT;
  const int i_start = p.causal ? k0 / KV_QT : 0;
  const int per_head = max(0, n_qt - i_start);
  const int n_it = rep * per_head;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int b = 0; b < KV_STAGES; ++b) {
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], KV_COMPUTE);
    }
    mbar_init(p_full, KV_COMPUTE);
    mbar_init(mma_done, 1);
    mbar_init(acc_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---------------------------------------------------------------- producer
    if (lane == 0 && n_it > 0) {
      mbar_arrive_expect_tx(kv_full, 2 * TILE_BYTES);
      tma_load_3d(sK, &tmK, kv_full, 0, kv_head, k_seg + k0);
      tma_load_3d(sK + HALF, &tmK, kv_full, 64, kv_head, k_seg + k0);
      tma_load_3d(sV, &tmV, kv_full, 0, kv_head, k_seg + k0);
      tma_load_3d(sV + HALF, &tmV, kv_full, 64, kv_head, k_seg + k0);
      int issued = 0;
      for (int it = 0; it < n_it; ++it) {
        const int s = it % KV_STAGES;
        if (it >= KV_STAGES &&
            !mbar_wait_bounded(&q_empty[s], (it / KV_STAGES - 1) & 1, abort_flag, p.status, kTimeoutProducer))
          break;
        const int h = kv_head * rep + it / per_head;
        const int i = i_start + it % per_head;
        int qrow = q_seg + i * KV_QT;
        const CUtensorMap* mq = &tmQ;
        const CUtensorMap* mo = &tmO;
        if constexpr (PEER) {
          int owner;
          qrow = peer_row(src, seq, i * KV_QT, owner);
          mq = &src.a[owner];
          mo = &src.b[owner];
        }
        uint8_t* dq = smem + KV_OFF_Q + s * KV_QBYTES;
        uint8_t* dd = smem + KV_OFF_DO + s * KV_QBYTES;
        mbar_arrive_expect_tx(&q_full[s], 2 * KV_QBYTES);
        tma_load_3d(dq, mq, &q_full[s], 0, h, qrow);
        tma_load_3d(dq + KV_QHALF, mq, &q_full[s], 64, h, qrow);
        tma_load_3d(dd, mo, &q_full[s], 0, h, qrow);
        tma_load_3d(dd + KV_QHALF, mo, &q_full[s], 64, h, qrow);
        issued = it + 1;
      }
      // copies still in flight after an abort land before the CTA exits
      mbar_wait_bounded(kv_full, 0, nullptr, nullptr, 0);
      for (int it = issued > KV_STAGES ? issued - KV_STAGES : 0; it < issued; ++it)
        mbar_wait_bounded(&q_full[it % KV_STAGES], (it / KV_STAGES) & 1, nullptr, nullptr, 0);
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && n_it > 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(128, KV_QT, 0, 0);   // K/V K-major x Q/dO K-major
      constexpr uint32_t idesc_g = make_idesc_bf16(128, 128, 0, 1);     // P^T/dS^T K-major x dO/Q MN-major
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aPT = smem_u32(sPT), adST = smem_u32(sdST);
      bool ok = mbar_wait_bounded(kv_full, 0, abort_flag, p.status, kTimeoutMma);
      for (int it = 0; ok && it <= n_it; ++it) {
        if (it < n_it) {
          const int s = it % KV_STAGES, b = it & 1;
          if (!mbar_wait_bounded(&q_full[s], (it / KV_STAGES) & 1, abort_flag, p.status, kTimeoutMma)) break;
          if (it >= 2 && !mbar_wait_bounded(&s_free[b], ((it >> 1) - 1) & 1, abort_flag, p.status, kTimeoutMma)) break;
          tc_fence_after();
          const uint32_t aQ = smem_u32(smem + KV_OFF_Q + s * KV_QBYTES);
          const uint32_t adO = smem_u32(smem + KV_OFF_DO + s * KV_QBYTES);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t bo = (k >> 2) * KV_QHALF + (k & 3) * 32;
            umma_bf16_ss(tmem + b * KV_QT, desc_kmajor(aK, k), make_smem_desc_sw128(aQ + bo, 16, 1024), idesc_s,
                         k > 0);
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t bo = (k >> 2) * KV_QHALF + (k & 3) * 32;
            umma_bf16_ss(tmem + 128 + b * KV_QT, desc_kmajor(aV, k), make_smem_desc_sw128(adO + bo, 16, 1024),
                         idesc_s, k > 0);
          }
          umma_commit(&s_full[b]);
        }
        if (it >= 1) {
          const int jt = it - 1, s = jt % KV_STAGES;
          if (!mbar_wait_bounded(p_full, jt & 1, abort_flag, p.status, kTimeoutMma)) break;
          tc_fence_after();
          const uint32_t aQ = smem_u32(smem + KV_OFF_Q + s * KV_QBYTES);
          const uint32_t adO = smem_u32(smem + KV_OFF_DO + s * KV_QBYTES);
#pragma unroll
          for (int k = 0; k < KV_QT / 16; ++k)
            umma_bf16_ss(tmem + 256, make_smem_desc_sw128(aPT + k * 32, 16, 1024),
                         make_smem_desc_sw128(adO + k * 2048, KV_QHALF, 1024), idesc_g, (jt > 0 || k > 0));
#pragma unroll
          for (int k = 0; k < KV_QT / 16; ++k)
            umma_bf16_ss(tmem + 384, make_smem_desc_sw128(adST + k * 32, 16, 1024),
                         make_smem_desc_sw128(aQ + k * 2048, KV_QHALF, 1024), idesc_g, (jt > 0 || k > 0));
          umma_commit(mma_done);
          umma_commit(&q_empty[s]);
        }
      }
      umma_commit(acc_done);
    }
  } else {
    // ---------------------------------------------------------------- P^T / dS^T rows
    const int r = threadIdx.x & 127;   // key row == TMEM lane
    const int half = threadIdx.x >> 7; // which 32 of the 64 query columns
    const int kk = k0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const float c_log2 = p.scale * kLog2e;
    const bool row_ok = kk < k_len;
    // LSE and D of a query tile: threads r < 64 of the first half load row r from global memory one
    // iteration ahead (the loads are in flight during the previous tile's math) and store it into the
    // shared double buffer [it & 1] at the end of that iteration.
    const bool stat_thread = half == 0 && r < KV_QT;
    auto fetch_stats = [&](int it2, float& l, float& d) {
      const int h = kv_head * rep + it2 / per_head;
      const int q0 = (i_start + it2 % per_head) * KV_QT;
      const int qq = q0 + r;
      const float* lse_src = p.lse;
      const float* dsum_src = p.dsum;
      long row = q_seg + qq;
      if constexpr (PEER) {
        int owner;
        row = peer_row(src, seq, q0, owner) + r;
        lse_src = src.lse[owner];
        dsum_src = src.dsum[owner];
      }
      const bool v = qq < q_len && PRISM_IN_BOUNDS(row, p.tq, p.status);
      l = v ? lse_src[(long)h * p.tq + row] * kLog2e : INFINITY;
      d = v ? dsum_src[(long)h * p.tq + row] : 0.f;
    };
    if (stat_thread && n_it > 0) {
      float l, d;
      fetch_stats(0, l, d);
      lse_s[r] = l;
      dsum_s[r] = d;
    }
    bool ok = true;
    for (int it = 0; it < n_it && ok; ++it) {
      const int b = it & 1;
      const int i = i_start + it % per_head;
      const int q0 = i * KV_QT;
      // the stats of tile it are in smem; every thread has finished reading those of tile it - 1
      named_sync_kv();
      float next_l = 0.f, next_d = 0.f;
      const bool prefetch = stat_thread && it + 1 < n_it;
      if (prefetch) fetch_stats(it + 1, next_l, next_d);
      ok = named_barrier_and(mbar_wait_bounded(&s_full[b], (it >> 1) & 1, abort_flag, p.status, kTimeoutEpilogue),
                             1, KV_COMPUTE);
      if (!ok) break;
      tc_fence_after();
      const int col0 = half * 32;
      uint32_t s_raw[32], dp_raw[32];
      tmem_ld_32x32b_x32(lane_base + b * KV_QT + col0, s_raw);
      tmem_ld_32x32b_x32(lane_base + 128 + b * KV_QT + col0, dp_raw);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_free[b]);
      // P^T and dS^T overwrite the loaded S^T / dP^T values in place (keeps register use flat); the
      // stats are read as float4 broadcasts
      const float4* lse4 = reinterpret_cast<const float4*>(lse_s + b * KV_QT + col0);
      const float4* dsum4 = reinterpret_cast<const float4*>(dsum_s + b * KV_QT + col0);
#pragma unroll
      for (int e4 = 0; e4 < 8; ++e4) {
        const float4 l4 = lse4[e4], d4 = dsum4[e4];
        const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dv[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = 4 * e4 + u;
          const int qq = q0 + col0 + e;
          const bool valid = row_ok && qq < q_len && (!p.causal || kk <= qq);
          const float pe = valid ? exp2f(__uint_as_float(s_raw[e]) * c_log2 - lv[u]) : 0.f;
          s_raw[e] = __float_as_uint(pe);
          dp_raw[e] = __float_as_uint(pe * (__uint_as_float(dp_raw[e]) - dv[u]));
        }
      }
      const float* pv = reinterpret_cast<const float*>(s_raw);
      const float* dsv = reinterpret_cast<const float*>(dp_raw);
      // P^T / dS^T of the previous query tile must have been consumed
      if (it > 0) {
        ok = named_barrier_and(mbar_wait_bounded(mma_done, (it - 1) & 1, abort_flag, p.status, kTimeoutEpilogue),
                               1, KV_COMPUTE);
        if (!ok) break;
      }
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int off = r * 128 + (((half * 4 + g) ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(sPT + off) =
            make_uint4(pack_bf16x2(pv[8 * g], pv[8 * g + 1]), pack_bf16x2(pv[8 * g + 2], pv[8 * g + 3]),
                       pack_bf16x2(pv[8 * g + 4], pv[8 * g + 5]), pack_bf16x2(pv[8 * g + 6], pv[8 * g + 7]));
        *reinterpret_cast<uint4*>(sdST + off) =
            make_uint4(pack_bf16x2(dsv[8 * g], dsv[8 * g + 1]), pack_bf16x2(dsv[8 * g + 2], dsv[8 * g + 3]),
                       pack_bf16x2(dsv[8 * g + 4], dsv[8 * g + 5]), pack_bf16x2(dsv[8 * g + 6], dsv[8 * g + 7]));
      }
      if (prefetch) {
        lse_s[(b ^ 1) * KV_QT + r] = next_l;
        dsum_s[(b ^ 1) * KV_QT + r] = next_d;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && n_it > 0) ok = mbar_wait_bounded(acc_done, 0, abort_flag, p.status, kTimeoutEpilogue);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    {
      // every thread of the warp takes part in tcgen05.ld; only rows inside the sequence store
      const bool store = kk < k_len && PRISM_IN_BOUNDS(k_seg + kk, p.tk, p.status);
      const bool loaded = __all_sync(0xffffffffu, n_it > 0 && ok);
      __nv_bfloat16* dv_row = p.out2 + (long)(k_seg + kk) * p.out_stride + (long)kv_head * D;
      __nv_bfloat16* dk_row = p.out + (long)(k_seg + kk) * p.out_stride + (long)kv_head * D;
#pragma unroll 1
      for (int c = 2 * half; c < 2 * half + 2; ++c) {  // each half of the compute warps stores 64 columns
        uint32_t a[32], bb[32];
        if (loaded) {
          tmem_ld_32x32b_x32(lane_base + 256 + c * 32, a);
          tmem_ld_32x32b_x32(lane_base + 384 + c * 32, bb);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) a[e] = bb[e] = 0u;
        }
        if (!store) continue;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          reinterpret_cast<uint4*>(dv_row + c * 32)[v] = make_uint4(
              pack_bf16x2(__uint_as_float(a[8 * v]), __uint_as_float(a[8 * v + 1])),
              pack_bf16x2(__uint_as_float(a[8 * v + 2]), __uint_as_float(a[8 * v + 3])),
              pack_bf16x2(__uint_as_float(a[8 * v + 4]), __uint_as_float(a[8 * v + 5])),
              pack_bf16x2(__uint_as_float(a[8 * v + 6]), __uint_as_float(a[8 * v + 7])));
          reinterpret_cast<uint4*>(dk_row + c * 32)[v] = make_uint4(
              pack_bf16x2(__uint_as_float(bb[8 * v]) * p.scale, __uint_as_float(bb[8 * v + 1]) * p.scale),
              pack_bf16x2(__uint_as_float(bb[8 * v + 2]) * p.scale, __uint_as_float(bb[8 * v + 3]) * p.scale),
              pack_bf16x2(__uint_as_float(bb[8 * v + 4]) * p.scale, __uint_as_float(bb[8 * v + 5]) * p.scale),
              pack_bf16x2(__uint_as_float(bb[8 * v + 6]) * p.scale, __uint_as_float(bb[8 * v + 7]) * p.scale));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ dQ
// Eight compute warps as in the dK/dV kernel (warps w and w + 4 split the 128 key columns of a tile),
// warp 8 the TMA producer, warp 9 the MMA issuer. The compute warps release S / dP as soon as they
// are in registers, so S and dP of the next key tile are computed while dS of this one is formed.
constexpr int Q_THREADS = 320;
constexpr int Q_COMPUTE = 256;

template <class Src>
__global__ void __launch_bounds__(Q_THREADS, 1)
    attn_bwd_q_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, Params p,
                      const __grid_constant__ Src src) {
  constexpr bool PEER = std::is_same<Src, PeerTiles>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sdO = smem + TILE_BYTES;
  uint8_t* sK = smem + 2 * TILE_BYTES;  // [2]
  uint8_t* sV = smem + 4 * TILE_BYTES;  // [2]
  uint8_t* sdS = smem + 6 * TILE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 7 * TILE_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* ds_full = bars + 6;
  uint64_t* acc_done = bars + 7;
  uint64_t* s_free = bars + 8;    // S / dP of the current tile are in the compute warps' registers
  uint64_t* ds_free = bars + 9;   // the dQ product has read the dS tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 11);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int kv_head = head / (p.hq / p.hkv);
  int seq, q0, q_seg, q_len, k_seg, k_len;
  if constexpr (PEER) {
    seq = p.tiles[3 * blockIdx.x];
    q0 = p.tiles[3 * blockIdx.x + 1];
    q_seg = p.tiles[3 * blockIdx.x + 2] - q0;
    q_len = k_len = src.seq_n[seq];
    k_seg = 0;
  } else {
    seq = p.tiles[2 * blockIdx.x];
    q0 = p.tiles[2 * blockIdx.x + 1] * TILE;
    q_seg = p.cu_q[seq];
    q_len = p.cu_q[seq + 1] - q_seg;
    k_seg = p.cu_k[seq];
    k_len = p.cu_k[seq + 1] - k_seg;
  }
  const int kv_end = p.causal ? min(k_len, q0 + TILE) : k_len;
  const int n_kv = kv_end > 0 ? (kv_end + TILE - 1) / TILE : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(ds_full, Q_COMPUTE);
    mbar_init(acc_done, 1);
    mbar_init(s_free, Q_COMPUTE);
    mbar_init(ds_free, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    if (lane == 0 && n_kv > 0) {
      mbar_arrive_expect_tx(q_full, 2 * TILE_BYTES);
      tma_load_3d(sQ, &tmQ, q_full, 0, head, q_seg + q0);
      tma_load_3d(sQ + HALF, &tmQ, q_full, 64, head, q_seg + q0);
      tma_load_3d(sdO, &tmO, q_full, 0, head, q_seg + q0);
      tma_load_3d(sdO + HALF, &tmO, q_full, 64, head, q_seg + q0);
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        if (!mbar_wait_bounded(&kv_empty[s], ((j >> 1) & 1) ^ 1, abort_flag, p.status, kTimeoutProducer)) break;
        mbar_arrive_expect_tx(&kv_full[s], 2 * TILE_BYTES);
        int krow = k_seg + j * TILE;
        const CUtensorMap* mk = &tmK;
        const CUtensorMap* mv = &tmV;
        if constexpr (PEER) {
          int owner;
          krow = peer_row(src, seq, j * TILE, owner);
          mk = &src.a[owner];
          mv = &src.b[owner];
        }
        uint8_t* kd = sK + s * TILE_BYTES;
        uint8_t* vd = sV + s * TILE_BYTES;
        tma_load_3d(kd, mk, &kv_full[s], 0, kv_head, krow);
        tma_load_3d(kd + HALF, mk, &kv_full[s], 64, kv_head, krow);
        tma_load_3d(vd, mv, &kv_full[s], 0, kv_head, krow);
        tma_load_3d(vd + HALF, mv, &kv_full[s], 64, kv_head, krow);
      }
    }
  } else if (warp == 9) {
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t idesc_kk = make_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idesc_km = make_idesc_bf16(128, 128, 0, 1);
      const uint32_t aQ = smem_u32(sQ), adO = smem_u32(sdO), adS = smem_u32(sdS);
      bool ok = mbar_wait_bounded(q_full, 0, abort_flag, p.status, kTimeoutMma);
      // step j issues S_j, dP_j (once the compute warps hold S_{j-1}, dP_{j-1} in registers), then
      // dQ += dS_{j-1} K_{j-1}
      for (int j = 0; ok && j <= n_kv; ++j) {
        if (j < n_kv) {
          const int s = j & 1;
          if (!mbar_wait_bounded(&kv_full[s], (j >> 1) & 1, abort_flag, p.status, kTimeoutMma)) break;
          if (j >= 1 && !mbar_wait_bounded(s_free, (j - 1) & 1, abort_flag, p.status, kTimeoutMma)) break;
          tc_fence_after();
          const uint32_t aK = smem_u32(sK + s * TILE_BYTES), aV = smem_u32(sV + s * TILE_BYTES);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            umma_bf16_ss(tmem + 0, desc_kmajor(aQ, k), desc_kmajor(aK, k), idesc_kk, k > 0);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            umma_bf16_ss(tmem + 128, desc_kmajor(adO, k), desc_kmajor(aV, k), idesc_kk, k > 0);
          umma_commit(s_full);
        }
        if (j >= 1) {
          const int jt = j - 1, s = jt & 1;
          if (!mbar_wait_bounded(ds_full, jt & 1, abort_flag, p.status, kTimeoutMma)) break;
          tc_fence_after();
          const uint32_t aK = smem_u32(sK + s * TILE_BYTES);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            umma_bf16_ss(tmem + 256, desc_kmajor(adS, k), desc_mnmajor(aK, k), idesc_km, (jt > 0 || k > 0));
          umma_commit(&kv_empty[s]);
          umma_commit(ds_free);
        }
      }
      umma_commit(acc_done);
    }
  } else {
    const int r = threadIdx.x & 127;
    const int half = threadIdx.x >> 7;   // which 64 of the tile's 128 key columns
    const int qq = q0 + r;
    const bool row_ok = qq < q_len && PRISM_IN_BOUNDS(q_seg + qq, p.tq, p.status);
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const float c_log2 = p.scale * kLog2e;
    const float lse2 = row_ok ? p.lse[(long)head * p.tq + q_seg + qq] * kLog2e : INFINITY;
    const float dsum = row_ok ? p.dsum[(long)head * p.tq + q_seg + qq] : 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv && ok; ++j) {
      // decided jointly by all 256 compute threads, so both halves of a row take the same path
      ok = named_barrier_and(mbar_wait_bounded(s_full, j & 1, abort_flag, p.status, kTimeoutEpilogue), 1, Q_COMPUTE);
      if (!ok) break;
      tc_fence_after();
      const int col0 = half * 64;
      uint32_t s_raw[64], dp_raw[64];
      tmem_ld_32x32b_x32(lane_base + col0, *reinterpret_cast<uint32_t(*)[32]>(s_raw));
      tmem_ld_32x32b_x32(lane_base + col0 + 32, *reinterpret_cast<uint32_t(*)[32]>(s_raw + 32));
      tmem_ld_32x32b_x32(lane_base + 128 + col0, *reinterpret_cast<uint32_t(*)[32]>(dp_raw));
      tmem_ld_32x32b_x32(lane_base + 128 + col0 + 32, *reinterpret_cast<uint32_t(*)[32]>(dp_raw + 32));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(s_free);
      const int kbase = j * TILE + col0;
#pragma unroll
      for (int e = 0; e < 64; ++e) {
        const int kk = kbase + e;
        const bool valid = row_ok && kk < k_len && (!p.causal || kk <= qq);
        const float pe = valid ? exp2f(__uint_as_float(s_raw[e]) * c_log2 - lse2) : 0.f;
        dp_raw[e] = __float_as_uint(pe * (__uint_as_float(dp_raw[e]) - dsum));
      }
      const float* dsv = reinterpret_cast<const float*>(dp_raw);
      // the dQ product of the previous tile must have read the dS tile before it is rewritten
      if (j >= 1) {
        ok = named_barrier_and(mbar_wait_bounded(ds_free, (j - 1) & 1, abort_flag, p.status, kTimeoutEpilogue),
                               1, Q_COMPUTE);
        if (!ok) break;
      }
#pragma unroll
      for (int g = 0; g < 8; ++g)
        write_chunk_sw128(sdS, r, half * 8 + g,
                          make_uint4(pack_bf16x2(dsv[8 * g], dsv[8 * g + 1]),
                                     pack_bf16x2(dsv[8 * g + 2], dsv[8 * g + 3]),
                                     pack_bf16x2(dsv[8 * g + 4], dsv[8 * g + 5]),
                                     pack_bf16x2(dsv[8 * g + 6], dsv[8 * g + 7])));
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(ds_full);
    }
    if (ok && n_kv > 0) ok = mbar_wait_bounded(acc_done, 0, abort_flag, p.status, kTimeoutEpilogue);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    {
      const bool loaded = __all_sync(0xffffffffu, n_kv > 0 && ok);
      __nv_bfloat16* dq_row = p.out + (long)(q_seg + qq) * p.out_stride + (long)head * D;
#pragma unroll 1
      for (int c = 2 * half; c < 2 * half + 2; ++c) {  // each half of the compute warps stores 64 columns
        uint32_t a[32];
        if (loaded) {
          tmem_ld_32x32b_x32(lane_base + 256 + c * 32, a);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) a[e] = 0u;
        }
        if (!row_ok) continue;
#pragma unroll
        for (int v = 0; v < 4; ++v)
          reinterpret_cast<uint4*>(dq_row + c * 32)[v] = make_uint4(
              pack_bf16x2(__uint_as_float(a[8 * v]) * p.scale, __uint_as_float(a[8 * v + 1]) * p.scale),
              pack_bf16x2(__uint_as_float(a[8 * v + 2]) * p.scale, __uint_as_float(a[8 * v + 3]) * p.scale),
              pack_bf16x2(__uint_as_float(a[8 * v + 4]) * p.scale, __uint_as_float(a[8 * v + 5]) * p.scale),
              pack_bf16x2(__uint_as_float(a[8 * v + 6]) * p.scale, __uint_as_float(a[8 * v + 7]) * p.scale));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// D[h, t] = sum_d dO[t, h, d] * O[t, h, d]   (one warp per (t, h))
__global__ void attn_bwd_dot_kernel(const __nv_bfloat16* __restrict__ dO, long dos, const __nv_bfloat16* __restrict__ O,
                                    long os, float* __restrict__ out, int T, int H) {
  const long w = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long)T * H) return;
  const long t = w / H;
  const int h = w % H;
  const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(dO + t * dos + (long)h * D) + lane * 2;
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(O + t * os + (long)h * D) + lane * 2;
  float acc = 0.f;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float2 x = __bfloat1622float2(a[e]);
    const float2 y = __bfloat1622float2(b[e]);
    acc += x.x * y.x + x.y * y.y;
  }
  acc = warp_sum(acc);
  if (lane == 0) out[(long)h * T + t] = acc;
}

constexpr int SMEM_KV = KV_OFF_BAR + 256 + 1024;
constexpr int SMEM_Q = 7 * TILE_BYTES + 256 + 1024;
static_assert(12 * 8 <= 256, "dQ barriers fit their shared-memory slot");

}  // namespace attnb

void attention_bwd_sm100(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& out,
                         const at::Tensor& lse, const at::Tensor& dout, const at::Tensor& cu_q, const at::Tensor& cu_k,
                         const at::Tensor& tiles_q, const at::Tensor& tiles_k, at::Tensor& dq, at::Tensor& dk,
                         at::Tensor& dv, bool causal, double softmax_scale, at::Tensor& status) {
  using namespace attnb;
  const c10::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int Tq = q.size(0), hq = q.size(1), hkv = k.size(1);
  TORCH_CHECK(dk.stride(0) == dv.stride(0), "attention bwd: dk/dv must share a row stride");
  at::Tensor dsum = at::empty({hq, Tq}, q.options().dtype(at::kFloat));
  {
    const long warps = (long)Tq * hq;
    if (warps > 0)
      attn_bwd_dot_kernel<<<(warps * 32 + 255) / 256, 256, 0, stream>>>(
          reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), dout.stride(0),
          reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()), out.stride(0), dsum.data_ptr<float>(), Tq, hq);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  CUtensorMap tq = make_head_map_128(q), tk = make_head_map_128(k), tv = make_head_map_128(v),
              tdo = make_head_map_128(dout);
  // the dK/dV kernel streams query tiles of KV_QT rows
  CUtensorMap tq64 = make_head_map(q, KV_QT), tdo64 = make_head_map(dout, KV_QT);
  Params p;
  p.cu_q = cu_q.data_ptr<int>();
  p.cu_k = cu_k.data_ptr<int>();
  p.hq = hq;
  p.hkv = hkv;
  p.causal = causal ? 1 : 0;
  p.scale = (float)softmax_scale;
  p.lse = lse.data_ptr<float>();
  p.dsum = dsum.data_ptr<float>();
  p.tq = Tq;
  p.tk = k.size(0);
  p.status = status.data_ptr<int>();
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kv_kernel<NoPeers>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        SMEM_KV));
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_q_kernel<NoPeers>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        SMEM_Q));
    configured = true;
  }
  if (tiles_k.size(0) > 0) {
    Params pk = p;
    pk.tiles = tiles_k.data_ptr<int>();
    pk.out = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
    pk.out2 = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
    pk.out_stride = dk.stride(0);
    attn_bwd_kv_kernel<NoPeers><<<dim3(tiles_k.size(0), hkv), KV_THREADS, SMEM_KV, stream>>>(tq64, tk, tv, tdo64,
                                                                                             pk, NoPeers{0});
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  if (tiles_q.size(0) > 0) {
    Params pq = p;
    pq.tiles = tiles_q.data_ptr<int>();
    pq.out = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
    pq.out2 = nullptr;
    pq.out_stride = dq.stride(0);
    attn_bwd_q_kernel<NoPeers><<<dim3(tiles_q.size(0), hq), Q_THREADS, SMEM_Q, stream>>>(tq, tk, tv, tdo, pq,
                                                                                          NoPeers{0});
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

// Context-parallel backward over a zigzag team (causal). *_peers: the team's
// buffers in symmetric memory, indexed by team rank: q/k/v/dout [T, H, 128]
// views, lse/dsum [hq, T] fp32 (dsum = rowsum(dO * O), computed beforehand by
// attention_bwd_dsum on every rank). tiles int32 [n, 3] = (seq, global position
// of the tile's first row, its local row), the same list for keys and queries.
void attention_bwd_peer(const std::vector<at::Tensor>& q_peers, const std::vector<at::Tensor>& k_peers,
                        const std::vector<at::Tensor>& v_peers, const std::vector<at::Tensor>& do_peers,
                        const std::vector<at::Tensor>& lse_peers, const std::vector<at::Tensor>& dsum_peers,
                        int64_t rank, const at::Tensor& tiles, const at::Tensor& seq_n, const at::Tensor& seq_row0,
                        at::Tensor& dq, at::Tensor& dk, at::Tensor& dv, double softmax_scale, at::Tensor& status) {
  using namespace attnb;
  const int cp = q_peers.size();
  TORCH_CHECK(cp >= 1 && cp <= kMaxPeers && (int)k_peers.size() == cp && (int)v_peers.size() == cp &&
                  (int)do_peers.size() == cp && (int)lse_peers.size() == cp && (int)dsum_peers.size() == cp,
              "attention_bwd_peer: one buffer per team rank (1..8)");
  TORCH_CHECK(dk.stride(0) == dv.stride(0), "attention bwd: dk/dv must share a row stride");
  const at::Tensor& q = q_peers[rank];
  const c10::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int Tq = q.size(0), hq = q.size(1), hkv = k_peers[rank].size(1);
  const int ntiles = tiles.size(0);
  if (ntiles == 0) return;
  Params p;
  p.cu_q = nullptr;
  p.cu_k = nullptr;
  p.hq = hq;
  p.hkv = hkv;
  p.causal = 1;
  p.scale = (float)softmax_scale;
  p.lse = lse_peers[rank].data_ptr<float>();
  p.dsum = dsum_peers[rank].data_ptr<float>();
  p.tq = Tq;
  p.tk = k_peers[rank].size(0);
  p.status = status.data_ptr<int>();
  p.tiles = tiles.data_ptr<int>();
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kv_kernel<PeerTiles>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        SMEM_KV));
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_q_kernel<PeerTiles>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        SMEM_Q));
    configured = true;
  }
  CUtensorMap tq = make_head_map_128(q), tk = make_head_map_128(k_peers[rank]),
              tv = make_head_map_128(v_peers[rank]), tdo = make_head_map_128(do_peers[rank]);
  PeerTiles kv_src{}, q_src{};
  for (int r = 0; r < cp; ++r) {
    kv_src.a[r] = make_head_map(q_peers[r], KV_QT);
    kv_src.b[r] = make_head_map(do_peers[r], KV_QT);
    kv_src.lse[r] = lse_peers[r].data_ptr<float>();
    kv_src.dsum[r] = dsum_peers[r].data_ptr<float>();
    q_src.a[r] = make_head_map_128(k_peers[r]);
    q_src.b[r] = make_head_map_128(v_peers[r]);
  }
  kv_src.seq_n = q_src.seq_n = seq_n.data_ptr<int>();
  kv_src.seq_row0 = q_src.seq_row0 = seq_row0.data_ptr<int>();
  kv_src.cp = q_src.cp = cp;
  Params pk = p;
  pk.out = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  pk.out2 = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  pk.out_stride = dk.stride(0);
  CUtensorMap tq64 = make_head_map(q, KV_QT), tdo64 = make_head_map(do_peers[rank], KV_QT);
  attn_bwd_kv_kernel<PeerTiles><<<dim3(ntiles, hkv), KV_THREADS, SMEM_KV, stream>>>(tq64, tk, tv, tdo64, pk,
                                                                                     kv_src);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  Params pq = p;
  pq.out = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
  pq.out2 = nullptr;
  pq.out_stride = dq.stride(0);
  attn_bwd_q_kernel<PeerTiles><<<dim3(ntiles, hq), Q_THREADS, SMEM_Q, stream>>>(tq, tk, tv, tdo, pq, q_src);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// D = rowsum(dO * O) per (query, head): [hq, T] fp32.
void attention_bwd_dsum(const at::Tensor& out, const at::Tensor& dout, at::Tensor& dsum) {
  using namespace attnb;
  const c10::cuda::CUDAGuard guard(out.device());
  const int Tq = out.size(0), hq = out.size(1);
  const long warps = (long)Tq * hq;
  if (warps > 0)
    attn_bwd_dot_kernel<<<(warps * 32 + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), dout.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()), out.stride(0), dsum.data_ptr<float>(), Tq, hq);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace prism
