// Variable-length causal / full GQA flash-attention forward on tcgen05 (sm_100a).
//
// One CTA computes one 128-query tile of one query head (head_dim 128):
//   warps 0-7  softmax: query row r of the tile is TMEM lane r; warps w and w + 4
//              both own rows 32(w % 4).. and take one 64-key half of each score
//              row (after tcgen05.ld, no shuffles; the two halves exchange their
//              row maxima through shared memory). P = exp2(s - m) is written to
//              shared memory in the 128-byte-swizzled K-major layout the tensor
//              core reads as the A operand of P.V. The running max is only moved
//              (and O in TMEM rescaled) when it grows by more than 2^8, which keeps
//              the fp32 accumulators exact while making rescales rare.
//   warp 8     TMA producer: Q once, then K/V tiles of 128 keys into a 2-stage ring.
//   warp 9     allocates TMEM (S double buffer: cols 0-255, O: cols 256-383) and
//              issues S_j = Q K_j^T and O += P_{j-1} V_{j-1} from one thread.
// Q, K, V are read through 3-D tensor maps over [tokens, heads, 128] views with
// arbitrary token stride, so the kernel consumes the fused QKV projection in place.
// Causal masking is top-left aligned within a sequence (query i sees keys <= i),
// which is what the zigzag ring needs on its diagonal steps. Outputs: O (bf16)
// and the natural-log LSE per (query, head) for the backward and ring merges.
#include <cudaTypedefs.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tma_host.cuh"
#include "attention_peer.cuh"

#include <type_traits>

namespace prism {
namespace attn {

constexpr int D = 128;
constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int KV_STAGES = 2;
constexpr int TILE_BYTES = 128 * D * 2;  // 32 KiB: 128 rows x 128 dims (two 64-dim boxes)
// Eight softmax warps: warps w and w + 4 share TMEM lanes (query rows) 32(w % 4).. and split each
// 128-key tile into two 64-column halves, exchanging their row maxima through shared memory, so
// every SM sub-partition interleaves two warps of exponentials. Warp 8 is the TMA producer, warp 9
// allocates TMEM and issues the MMAs.
constexpr int NUM_THREADS = 320;
constexpr int SOFTMAX_THREADS = 256;
constexpr int TMEM_COLS = 512;
constexpr int TMEM_O = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
// smem: Q | K[2] | V[2] | P | barriers
constexpr int SMEM_Q = 0;
constexpr int SMEM_K = SMEM_Q + TILE_BYTES;
constexpr int SMEM_V = SMEM_K + KV_STAGES * TILE_BYTES;
constexpr int SMEM_P = SMEM_V + KV_STAGES * TILE_BYTES;
constexpr int SMEM_BAR = SMEM_P + TILE_BYTES;
constexpr int SMEM_XMAX = SMEM_BAR + 256;              // [3 buffers][2 halves][128 rows] fp32
constexpr int SMEM_BYTES = SMEM_XMAX + 3 * 2 * BQ * 4 + 1024;

struct FwdParams {
  const int* cu_q;      // [nseq+1]
  const int* cu_k;      // [nseq+1]
  const int* tiles;     // [ntiles*2]: (seq, q tile index within seq)
  int ntiles;
  int hq, hkv;
  int causal;
  float scale_log2;     // softmax scale * log2(e)
  __nv_bfloat16* out;   // [Tq, hq, 128] with row stride out_stride
  long out_stride;
  float* lse;           // [hq, Tq]   (natural log)
  int tq;
  int* status;
};

__device__ __forceinline__ void write_p_chunk(uint8_t* p_base, int row, int chunk, uint4 val) {
  // chunk: 0..15 (8 keys each). Two 64-key blocks of 128 rows x 128 B, 128-byte swizzle.
  const int blk = chunk >> 3, cc = chunk & 7;
  uint8_t* addr = p_base + blk * (128 * 128) + row * 128 + ((cc ^ (row & 7)) << 4);
  *reinterpret_cast<uint4*>(addr) = val;
}

// Src = NoPeers: K/V of the sequence are local (tiles hold (seq, q tile)).
// Src = PeerTiles: the sequence is spread over a zigzag team; tiles hold
// (seq, global position of the first query, its local row) and every KV tile is
// loaded from the rank that owns it.
template <class Src>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, FwdParams p, const __grid_constant__ Src src) {
  constexpr bool PEER = std::is_same<Src, PeerTiles>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SMEM_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;       // [2]
  uint64_t* kv_empty = bars + 3;      // [2]
  uint64_t* s_full = bars + 5;        // [2]
  uint64_t* s_free = bars + 7;        // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* pv_done = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 13);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int kv_head = head / (p.hq / p.hkv);
  int seq, q0, q_seg, q_len, k_seg, k_len;
  if constexpr (PEER) {
    seq = p.tiles[3 * blockIdx.x];
    q0 = p.tiles[3 * blockIdx.x + 1];              // global position within the sequence
    q_seg = p.tiles[3 * blockIdx.x + 2] - q0;      // local row = q_seg + position (this tile's rows)
    q_len = k_len = src.seq_n[seq];
    k_seg = 0;
  } else {
    seq = p.tiles[2 * blockIdx.x];
    q0 = p.tiles[2 * blockIdx.x + 1] * BQ;         // within the sequence
    q_seg = p.cu_q[seq];
    q_len = p.cu_q[seq + 1] - q_seg;
    k_seg = p.cu_k[seq];
    k_len = p.cu_k[seq + 1] - k_seg;
  }
  int kv_end = k_len;
  if (p.causal) kv_end = min(k_len, q0 + BQ);
  const int n_kv = kv_end > 0 ? (kv_end + BKV - 1) / BKV : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], SOFTMAX_THREADS);
    }
    mbar_init(p_full, SOFTMAX_THREADS);
    mbar_init(pv_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---------------------------------------------------------------- producer
    if (lane == 0 && n_kv > 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, TILE_BYTES);
      tma_load_3d(smem + SMEM_Q, &tmQ, q_full, 0, head, q_seg + q0);
      tma_load_3d(smem + SMEM_Q + TILE_BYTES / 2, &tmQ, q_full, 64, head, q_seg + q0);
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait_bounded(&kv_empty[s], ph ^ 1, abort_flag, p.status, kTimeoutProducer)) break;
        mbar_arrive_expect_tx(&kv_full[s], 2 * TILE_BYTES);
        int krow = k_seg + j * BKV;
        const CUtensorMap* mk = &tmK;
        const CUtensorMap* mv = &tmV;
        if constexpr (PEER) {
          int owner;
          krow = peer_row(src, seq, j * BKV, owner);
          mk = &src.a[owner];
          mv = &src.b[owner];
        }
        uint8_t* kd = smem + SMEM_K + s * TILE_BYTES;
        uint8_t* vd = smem + SMEM_V + s * TILE_BYTES;
        tma_load_3d(kd, mk, &kv_full[s], 0, kv_head, krow);
        tma_load_3d(kd + TILE_BYTES / 2, mk, &kv_full[s], 64, kv_head, krow);
        tma_load_3d(vd, mv, &kv_full[s], 0, kv_head, krow);
        tma_load_3d(vd + TILE_BYTES / 2, mv, &kv_full[s], 64, kv_head, krow);
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(128, 128, 0, 0);  // Q,K both K-major (dim contiguous)
      constexpr uint32_t idesc_o = make_idesc_bf16(128, 128, 0, 1);  // P K-major, V MN-major
      const uint32_t q_addr = smem_u32(smem + SMEM_Q);
      const uint32_t p_addr = smem_u32(smem + SMEM_P);
      bool ok = mbar_wait_bounded(q_full, 0, abort_flag, p.status, kTimeoutMma);
      for (int j = 0; ok && j <= n_kv; ++j) {
        if (j < n_kv) {
          const int s = j & 1;
          const uint32_t ph = (j >> 1) & 1;
          if (!mbar_wait_bounded(&kv_full[s], ph, abort_flag, p.status, kTimeoutMma)) break;
          if (!mbar_wait_bounded(&s_free[s], ph ^ 1, abort_flag, p.status, kTimeoutMma)) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(smem + SMEM_K + s * TILE_BYTES);
          const uint32_t d_tmem = tmem + s * 128;
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t off = (k >> 2) * (TILE_BYTES / 2) + (k & 3) * 32;
            umma_bf16_ss(d_tmem, make_smem_desc_sw128(q_addr + off, 16, 1024),
                         make_smem_desc_sw128(k_addr + off, 16, 1024), idesc_s, k > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[s]);
        }
        if (j > 0) {
          const int jp = j - 1;
          const int s = jp & 1;
          if (!mbar_wait_bounded(p_full, jp & 1, abort_flag, p.status, kTimeoutMma)) break;
          tc_fence_after();
          const uint32_t v_addr = smem_u32(smem + SMEM_V + s * TILE_BYTES);
#pragma unroll
          for (int k = 0; k < BKV / 16; ++k) {
            const uint32_t a_off = (k >> 2) * (128 * 128) + (k & 3) * 32;
            umma_bf16_ss(tmem + TMEM_O, make_smem_desc_sw128(p_addr + a_off, 16, 1024),
                         make_smem_desc_sw128(v_addr + k * 2048, TILE_BYTES / 2, 1024), idesc_o,
                         (jp > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(pv_done);
          umma_commit(&kv_empty[s]);
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax
    const int r = threadIdx.x & 127;  // 0..127 == TMEM lane
    const int half = threadIdx.x >> 7;
    const int col0 = half * 64;       // this thread's 64 keys of each tile
    const int q_idx = q0 + r;         // within sequence
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    float* xmax = reinterpret_cast<float*>(smem + SMEM_XMAX);  // [buffer][half][row]
    float m = -INFINITY;  // running max in log2 units (identical in both halves of a row)
    float l = 0.f;        // this half's share of the row sum
    uint8_t* p_base = smem + SMEM_P;
    bool ok = true;
    for (int j = 0; j < n_kv && ok; ++j) {
      const int s = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      // every wait is decided per warp, then jointly by all 256 softmax threads at the one named
      // barrier of the iteration, so both halves of a row always take the same path
      const bool got = __all_sync(0xffffffffu,
                                  mbar_wait_bounded(&s_full[s], ph, abort_flag, p.status, kTimeoutEpilogue));
      float sv[64];
      if (got) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t raw[32];
          tmem_ld_32x32b_x32(lane_base + s * 128 + col0 + c * 32, raw);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) sv[c * 32 + e] = __uint_as_float(raw[e]) * p.scale_log2;
        }
        tc_fence_before();
        mbar_arrive(&s_free[s]);
      } else {
#pragma unroll
        for (int e = 0; e < 64; ++e) sv[e] = -INFINITY;
      }
      // masking
      const int k_base = j * BKV + col0;
      const bool need_mask = (k_base + 64 > k_len) || (p.causal && k_base + 63 > q0) || (q_idx >= q_len);
      if (need_mask) {
#pragma unroll
        for (int e = 0; e < 64; ++e) {
          const int kk = k_base + e;
          const bool valid = kk < k_len && q_idx < q_len && (!p.causal || kk <= q_idx);
          if (!valid) sv[e] = -INFINITY;
        }
      }
      float hmax = sv[0];
#pragma unroll
      for (int e = 1; e < 64; ++e) hmax = fmaxf(hmax, sv[e]);
      // P_j may only be written after PV_{j-1} finished reading P_{j-1}
      const bool pv_ok = j == 0 || __all_sync(0xffffffffu, mbar_wait_bounded(pv_done, (j - 1) & 1, abort_flag,
                                                                              p.status, kTimeoutEpilogue));
      // the row maximum over both halves (a double buffer: a half can be one tile ahead)
      xmax[(s * 2 + half) * BQ + r] = hmax;
      ok = named_barrier_and(got && pv_ok, 1, SOFTMAX_THREADS);
      if (!ok) break;
      const float tmax = fmaxf(hmax, xmax[(s * 2 + (half ^ 1)) * BQ + r]);
      float alpha = 1.f;
      if (tmax > m + kRescaleThreshold || (m == -INFINITY && tmax > -INFINITY)) {
        const float m_new = fmaxf(tmax, m);
        alpha = (m == -INFINITY) ? 0.f : exp2f(m - m_new);
        m = m_new;
      }
      const float mm = (m == -INFINITY) ? 0.f : m;
      float rowsum = 0.f;
      // tcgen05.ld/st are warp-collective (.sync.aligned): the rescale runs for the whole warp
      // whenever any of its rows needs it (rows that do not multiply by alpha = 1); each half
      // rescales its own 64 of the 128 output columns
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t raw[32];
          tmem_ld_32x32b_x32(lane_base + TMEM_O + col0 + c * 32, raw);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) raw[e] = __float_as_uint(__uint_as_float(raw[e]) * alpha);
          tmem_st_32x32b_x32(lane_base + TMEM_O + col0 + c * 32, raw);
        }
        tmem_wait_st();
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float pe[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          pe[e] = exp2f(sv[c * 8 + e] - mm);
          rowsum += pe[e];
        }
        const uint4 packed = make_uint4(pack_bf16x2(pe[0], pe[1]), pack_bf16x2(pe[2], pe[3]),
                                        pack_bf16x2(pe[4], pe[5]), pack_bf16x2(pe[6], pe[7]));
        write_p_chunk(p_base, r, half * 8 + c, packed);
      }
      l = l * alpha + rowsum;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // epilogue: the row sum is the two halves' shares (its own buffer: the other half may still be
    // reading the last tile's maxima)
    xmax[(4 + half) * BQ + r] = l;
    ok = named_barrier_and(ok, 1, SOFTMAX_THREADS);
    l += xmax[(4 + (half ^ 1)) * BQ + r];
    if (ok && n_kv > 0) ok = mbar_wait_bounded(pv_done, (n_kv - 1) & 1, abort_flag, p.status, kTimeoutEpilogue);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const bool row_valid = q_idx < q_len && PRISM_IN_BOUNDS(q_seg + q_idx, p.tq, p.status);
    const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
    __nv_bfloat16* orow = p.out + (long)(q_seg + q_idx) * p.out_stride + (long)head * D;
#pragma unroll
    for (int c = 2 * half; c < 2 * half + 2; ++c) {
      uint32_t raw[32];
      if (n_kv > 0 && ok) {
        tmem_ld_32x32b_x32(lane_base + TMEM_O + c * 32, raw);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) raw[e] = 0u;
      }
      if (row_valid) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const uint4 packed = make_uint4(
              pack_bf16x2(__uint_as_float(raw[8 * v + 0]) * inv_l, __uint_as_float(raw[8 * v + 1]) * inv_l),
              pack_bf16x2(__uint_as_float(raw[8 * v + 2]) * inv_l, __uint_as_float(raw[8 * v + 3]) * inv_l),
              pack_bf16x2(__uint_as_float(raw[8 * v + 4]) * inv_l, __uint_as_float(raw[8 * v + 5]) * inv_l),
              pack_bf16x2(__uint_as_float(raw[8 * v + 6]) * inv_l, __uint_as_float(raw[8 * v + 7]) * inv_l));
          reinterpret_cast<uint4*>(orow + c * 32)[v] = packed;
        }
      }
    }
    if (row_valid && half == 0) {
      const float lse = (l > 0.f) ? (m + log2f(l)) * 0.69314718055994530942f : -INFINITY;
      p.lse[(long)head * p.tq + q_seg + q_idx] = lse;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace attn

// q [Tq,Hq,128], k/v [Tk,Hkv,128] (views), cu_q/cu_k int32 device [nseq+1], tiles int32 device [ntiles,2].
void attention_fwd_sm100(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& cu_q,
                         const at::Tensor& cu_k, const at::Tensor& tiles, at::Tensor& out, at::Tensor& lse,
                         bool causal, double softmax_scale, at::Tensor& status) {
  using namespace attn;
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
              "attention: bf16");
  TORCH_CHECK(out.dim() == 3 && out.stride(2) == 1 && out.stride(1) == D, "attention: out [T,H,128]");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous(), "attention: lse fp32 [H,T]");
  const int hq = q.size(1), hkv = k.size(1);
  TORCH_CHECK(hq % hkv == 0, "attention: query heads must be a multiple of kv heads");
  const int ntiles = tiles.size(0);
  if (ntiles == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  CUtensorMap tq = make_head_map_128(q), tk = make_head_map_128(k), tv = make_head_map_128(v);
  FwdParams p;
  p.cu_q = cu_q.data_ptr<int>();
  p.cu_k = cu_k.data_ptr<int>();
  p.tiles = tiles.data_ptr<int>();
  p.ntiles = ntiles;
  p.hq = hq;
  p.hkv = hkv;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = (float)(softmax_scale * 1.4426950408889634);
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.out_stride = out.stride(0);
  p.lse = lse.data_ptr<float>();
  p.tq = q.size(0);
  p.status = status.data_ptr<int>();
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<NoPeers>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        SMEM_BYTES));
    configured = true;
  }
  dim3 grid(ntiles, hq);
  attn_fwd_kernel<NoPeers><<<grid, NUM_THREADS, SMEM_BYTES, at::cuda::getCurrentCUDAStream()>>>(tq, tk, tv, p,
                                                                                                  NoPeers{0});
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Causal attention of this rank's zigzag query rows over a whole team's keys.
// k_peers / v_peers: the team's K / V buffers ([Tk, Hkv, 128] views, this rank's
// included, indexed by team rank) in symmetric memory; tiles int32 [n, 3] =
// (seq, global position of the first query, local row); seq_n / seq_row0 int32 [nseq].
void attention_fwd_peer(const at::Tensor& q, const std::vector<at::Tensor>& k_peers,
                        const std::vector<at::Tensor>& v_peers, const at::Tensor& tiles, const at::Tensor& seq_n,
                        const at::Tensor& seq_row0, at::Tensor& out, at::Tensor& lse, double softmax_scale,
                        at::Tensor& status) {
  using namespace attn;
  const int cp = k_peers.size();
  TORCH_CHECK(cp >= 1 && cp <= kMaxPeers && (int)v_peers.size() == cp, "attention_fwd_peer: 1..8 peers");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16, "attention: bf16");
  TORCH_CHECK(out.dim() == 3 && out.stride(2) == 1 && out.stride(1) == D, "attention: out [T,H,128]");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous(), "attention: lse fp32 [H,T]");
  const int hq = q.size(1), hkv = k_peers[0].size(1);
  TORCH_CHECK(hq % hkv == 0, "attention: query heads must be a multiple of kv heads");
  const int ntiles = tiles.size(0);
  if (ntiles == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  CUtensorMap tq = make_head_map_128(q);
  PeerTiles src{};
  for (int r = 0; r < cp; ++r) {
    src.a[r] = make_head_map_128(k_peers[r]);
    src.b[r] = make_head_map_128(v_peers[r]);
  }
  src.seq_n = seq_n.data_ptr<int>();
  src.seq_row0 = seq_row0.data_ptr<int>();
  src.cp = cp;
  FwdParams p;
  p.cu_q = nullptr;
  p.cu_k = nullptr;
  p.tiles = tiles.data_ptr<int>();
  p.ntiles = ntiles;
  p.hq = hq;
  p.hkv = hkv;
  p.causal = 1;
  p.scale_log2 = (float)(softmax_scale * 1.4426950408889634);
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.out_stride = out.stride(0);
  p.lse = lse.data_ptr<float>();
  p.tq = q.size(0);
  p.status = status.data_ptr<int>();
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<PeerTiles>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        SMEM_BYTES));
    configured = true;
  }
  dim3 grid(ntiles, hq);
  attn_fwd_kernel<PeerTiles><<<grid, NUM_THREADS, SMEM_BYTES, at::cuda::getCurrentCUDAStream()>>>(
      tq, src.a[0], src.b[0], p, src);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace prism
