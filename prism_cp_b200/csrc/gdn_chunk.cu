// Fused chunked gated delta rule for sm_100a (dk = 128, dv a multiple of 128).
//
// Per head, chunk of C = 64 tokens, with G = in-chunk cumsum of the log decay g,
// s = scale, E_ij = exp(G_i - G_j) and T = (I + L)^-1, L_ij = beta_i E_ij k_i.k_j (i > j):
//
//   Wn  = -T (beta e^G K)        U   = T (beta V)          (WY form)
//   Kd  = e^(G_last - G) K       Qg  = e^G s Q             gamma = e^(G_last)
//   Aqk = tril((s Q K^T) o E)
//   Delta_c = U_c + Wn_c S_c     S_{c+1} = gamma_c S_c + Kd_c^T Delta_c
//   O_c     = Qg_c S_c + Aqk_c Delta_c
//
// Kernels (one launch each, in this order):
//   gdn_prep_tc_kernel     tcgen05, one CTA per (chunk, head): G, KK^T and QK^T on
//                          the tensor cores, T = (I + L)^-1 by forward substitution,
//                          W and U as T-products on the tensor cores, Kd, Qg, Aqk.
//   gdn_state_tc_kernel<0> tcgen05, one CTA per (sequence, head, 128 columns of dv):
//                          the sequential state pass with the output fused in. The
//                          state is held TRANSPOSED in tensor memory (lane = value
//                          column v, 128 fp32 columns = dk), so every product of the
//                          recurrence is an M = 128 MMA:
//                            Delta^T = U^T + S^T Wn^T      (A = S^T bf16, B = Wn  K-major;
//                                                           U^T added as U^T x I on the tensor cores)
//                            S^T    <- gamma S^T + Delta^T Kd (A = Delta^T, B = Kd MN-major)
//                            O^T     = S^T Qg^T + Delta^T Aqk^T
//   gdn_state_tc_kernel<1> the reverse pass for the gradient G = dL/dS_{c+1}:
//                            dDelta^T = G^T Kd^T + dO^T Aqk
//                            G^T     <- gamma G^T + dO^T Qg + dDelta^T Wn
//   gdn_bwd_dv_kernel      tcgen05, one CTA per (chunk, head): every product that
//                          contracts over dv (dWn, dKd, dQg, dAqk, dDelta V^T, dgamma);
//                          a second launch can add the products of another state pass
//                          over the same chunks (the identity pass of GDN CP).
//   gdn_bwd_local_tc_kernel tcgen05, one CTA per (chunk, head): the WY backward, decay
//                          gradients and dq, dk, dv, dg, dbeta, every product on the
//                          tensor cores (gdn_bwd_local_kernel: the same on CUDA cores,
//                          kept as the reference form behind PRISM_GDN_LOCAL_TC=0).
// Sequences are padded to whole chunks (padded rows have q = k = v = 0, g = beta = 0,
// which leave the state unchanged). Every mbarrier wait is bounded; a kernel that
// gives up records an error code in the status word and returns.
#include <cstdlib>
#include <cstring>

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tma_host.cuh"

namespace prism {
namespace gdnc {

constexpr int C = 64;
constexpr int DK = 128;
constexpr int BLK = 64 * 128;  // one 128-byte-swizzled block of 64 rows x 64 bf16

PRISM_DEVICE uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

PRISM_DEVICE void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Byte offset of 16-byte chunk `cc` (8 bf16) of row `r` inside a 128-byte-swizzled block.
PRISM_DEVICE int swz(int r, int cc) { return r * 128 + ((cc ^ (r & 7)) << 4); }

PRISM_DEVICE float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }

PRISM_DEVICE void unpack8(uint4 u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

PRISM_DEVICE uint4 pack8(const float* f) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

PRISM_DEVICE uint4 pack8u(const uint32_t* r) {
  return make_uint4(pack_bf16x2(__uint_as_float(r[0]), __uint_as_float(r[1])),
                    pack_bf16x2(__uint_as_float(r[2]), __uint_as_float(r[3])),
                    pack_bf16x2(__uint_as_float(r[4]), __uint_as_float(r[5])),
                    pack_bf16x2(__uint_as_float(r[6]), __uint_as_float(r[7])));
}

// ============================================================================ shared loaders
constexpr int KP = DK + 1;  // fp32 row pitch of the k/q tiles (odd: conflict-free column reads)
constexpr int LP = 68;      // fp32 row pitch of L (multiple of 4: float4 row reads)

// Loads k (and q * scale) of one chunk as fp32 rows, zero rows past the end, plus
// g/beta; returns after the in-chunk cumulative sum G is in Gs.
PRISM_DEVICE void load_chunk_kq(const __nv_bfloat16* q, const __nv_bfloat16* k, const float* g, const float* beta,
                                int t0, int n, int h, int H, float scale, float* ks, float* qs, float* Gs,
                                float* Bs) {
  const int tid = threadIdx.x;
  for (int e = tid; e < C * (DK / 8); e += blockDim.x) {
    const int i = e / (DK / 8), a8 = (e % (DK / 8)) * 8;
    float kf[8], qf[8];
    if (i < n) {
      const long off = ((long)(t0 + i) * H + h) * DK + a8;
      unpack8(*reinterpret_cast<const uint4*>(k + off), kf);
      unpack8(*reinterpret_cast<const uint4*>(q + off), qf);
    } else {
#pragma unroll
      for (int m = 0; m < 8; ++m) kf[m] = qf[m] = 0.f;
    }
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      ks[i * KP + a8 + m] = kf[m];
      qs[i * KP + a8 + m] = qf[m] * scale;
    }
  }
  if (tid < 32) {
    float x0 = tid < n ? g[(long)(t0 + tid) * H + h] : 0.f;
    float x1 = tid + 32 < n ? g[(long)(t0 + tid + 32) * H + h] : 0.f;
    Bs[tid] = tid < n ? beta[(long)(t0 + tid) * H + h] : 0.f;
    Bs[tid + 32] = tid + 32 < n ? beta[(long)(t0 + tid + 32) * H + h] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y0 = __shfl_up_sync(0xffffffffu, x0, o);
      const float y1 = __shfl_up_sync(0xffffffffu, x1, o);
      if (tid >= o) {
        x0 += y0;
        x1 += y1;
      }
    }
    x1 += __shfl_sync(0xffffffffu, x0, 31);
    Gs[tid] = x0;
    Gs[tid + 32] = x1;
  }
  __syncthreads();
}

// ============================================================================ prep (tcgen05)
// One CTA (4 warps) per (chunk, head). K/Q/V tiles arrive by TMA; KK^T and
// QK^T are one M = 128 MMA each (rows 64..127 of the A operand read the next
// tile and land in TMEM lanes that are never read). Warps 0-1 (TMEM lanes =
// chunk rows) form L and Aqk, then solve T = (I + L)^-1 one column per thread
// and store T diag(beta e^G) and T diag(beta) in bf16 as A operands; the WY
// products W = T diag(beta e^G) K and U = T diag(beta) V are two more MMAs.
// Warps 2-3 write Kd and Qg meanwhile.
constexpr int TP_THREADS = 128;
constexpr int TP_TMEM_COLS = 512;  // [0,64) KK^T, [64,128) QK^T, [128,256) W, [256,256+DV) U

struct PrepTcParams {
  const float* g;
  const float* beta;
  const int* tok0;
  const int* len;
  __nv_bfloat16* Wn;
  __nv_bfloat16* U;
  __nv_bfloat16* Kd;
  __nv_bfloat16* Qg;
  __nv_bfloat16* Aqk;
  float* gam;
  float* Gc;
  float* aux;  // optional [Nc * H, 3, C, C] fp32: k_i.k_j, s q_i.k_j and T, for the backward
  float scale;
  int H, DV;
  int* status;
};

// The kernel allocates all 512 TMEM columns; its shared-memory request is raised so that two CTAs
// never share an SM (a second CTA would sit in tcgen05.alloc until the first one exits).
constexpr int kOneCtaPerSmSmem = 120 * 1024;
__host__ __device__ constexpr int prep_tc_smem(int DV) {
  return (6 + DV / 64) * BLK + C * LP * 4 + 2 * C * 4 + 64 + 1024 > kOneCtaPerSmSmem
             ? (6 + DV / 64) * BLK + C * LP * 4 + 2 * C * 4 + 64 + 1024
             : kOneCtaPerSmSmem;
}

__global__ void __launch_bounds__(TP_THREADS, 1)
    gdn_prep_tc_kernel(const __grid_constant__ CUtensorMap mQ, const __grid_constant__ CUtensorMap mK,
                       const __grid_constant__ CUtensorMap mV, PrepTcParams a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int DV = a.DV, H = a.H, nvb = DV / 64;
  uint8_t* sK = smem;
  uint8_t* sQ = sK + 2 * BLK;
  uint8_t* sV = sQ + 2 * BLK;
  uint8_t* sTk = sV + nvb * BLK;
  uint8_t* sTv = sTk + BLK;
  float* Ls = reinterpret_cast<float*>(sTv + BLK);
  float* Gs = Ls + C * LP;
  float* Bs = Gs + C;
  uint64_t* bars = reinterpret_cast<uint64_t*>(Bs + C);
  uint64_t* full = bars;
  uint64_t* mma1 = bars + 1;
  uint64_t* mma2 = bars + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
  const int ch = blockIdx.x, c = ch / H, h = ch % H;
  const int t0 = a.tok0[c], n = a.len[c];
  const int tid = threadIdx.x, warp = tid >> 5;

  if (tid == 0) {
    mbar_init(full, 1);
    mbar_init(mma1, 1);
    mbar_init(mma2, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, TP_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (tid == 0) {
    mbar_arrive_expect_tx(full, (4 + nvb) * BLK);
    tma_load_2d(sK, &mK, full, h * DK, t0);
    tma_load_2d(sK + BLK, &mK, full, h * DK + 64, t0);
    tma_load_2d(sQ, &mQ, full, h * DK, t0);
    tma_load_2d(sQ + BLK, &mQ, full, h * DK + 64, t0);
    for (int b = 0; b < nvb; ++b) tma_load_2d(sV + b * BLK, &mV, full, h * DV + b * 64, t0);
  }
  if (warp == 0) {
    const int l = tid;
    float x0 = l < n ? a.g[(long)(t0 + l) * H + h] : 0.f;
    float x1 = l + 32 < n ? a.g[(long)(t0 + l + 32) * H + h] : 0.f;
    Bs[l] = l < n ? a.beta[(long)(t0 + l) * H + h] : 0.f;
    Bs[l + 32] = l + 32 < n ? a.beta[(long)(t0 + l + 32) * H + h] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y0 = __shfl_up_sync(0xffffffffu, x0, o);
      const float y1 = __shfl_up_sync(0xffffffffu, x1, o);
      if (l >= o) {
        x0 += y0;
        x1 += y1;
      }
    }
    x1 += __shfl_sync(0xffffffffu, x0, 31);
    Gs[l] = x0;
    Gs[l + 32] = x1;
  }
  bool ok = __syncthreads_and(mbar_wait_bounded(full, 0, nullptr, a.status, kTimeoutProducer));
  if (ok) {
    if (n < C) {
      // rows past the end of the sequence hold the next sequence's tokens: zero them
      const int nblk = 4 + nvb;
      const int per = (C - n) * 8;
      for (int e = tid; e < nblk * per; e += TP_THREADS) {
        const int b = e / per, rem = e % per;
        const int r = n + rem / 8, cc = rem % 8;
        *reinterpret_cast<uint4*>(smem + b * BLK + swz(r, cc)) = make_uint4(0, 0, 0, 0);
      }
    }
    fence_proxy_async();
  }
  __syncthreads();
  if (ok && tid == 0) {
    tc_fence_after();
    const uint32_t k_addr = smem_u32(sK), q_addr = smem_u32(sQ);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t off = (k >> 2) * BLK + (k & 3) * 32;
      umma_bf16_ss(tmem, make_smem_desc_sw128(k_addr + off, 16, 1024), make_smem_desc_sw128(k_addr + off, 16, 1024),
                   make_idesc_bf16(128, 64, 0, 0), k > 0);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t off = (k >> 2) * BLK + (k & 3) * 32;
      umma_bf16_ss(tmem + 64, make_smem_desc_sw128(q_addr + off, 16, 1024),
                   make_smem_desc_sw128(k_addr + off, 16, 1024), make_idesc_bf16(128, 64, 0, 0), k > 0);
    }
    umma_commit(mma1);
  }
  const float GL = Gs[C - 1];
  if (ok && warp >= 2) {
    // Kd = e^(G_last - G) k and Qg = e^G s q, one row per thread
    const int r = tid - 64;
    const float eg = __expf(Gs[r]) * a.scale, ed = __expf(GL - Gs[r]);
    __nv_bfloat16* kd = a.Kd + ((long)ch * C + r) * DK;
    __nv_bfloat16* qg = a.Qg + ((long)ch * C + r) * DK;
#pragma unroll 4
    for (int cc = 0; cc < 16; ++cc) {
      float fk[8], fq[8];
      unpack8(*reinterpret_cast<const uint4*>(sK + (cc >> 3) * BLK + swz(r, cc & 7)), fk);
      unpack8(*reinterpret_cast<const uint4*>(sQ + (cc >> 3) * BLK + swz(r, cc & 7)), fq);
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        fk[m] *= ed;
        fq[m] *= eg;
      }
      reinterpret_cast<uint4*>(kd)[cc] = pack8(fk);
      reinterpret_cast<uint4*>(qg)[cc] = pack8(fq);
    }
  }
  if (warp < 2) {
    const bool waited = __all_sync(0xffffffffu, ok && mbar_wait_bounded(mma1, 0, nullptr, a.status, kTimeoutEpilogue));
    if (waited) {
      tc_fence_after();
      const int i = tid;
      const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
      uint32_t kk[64], qk[64];
      tmem_ld_32x32b_x32(tl, *reinterpret_cast<uint32_t(*)[32]>(kk));
      tmem_ld_32x32b_x32(tl + 32, *reinterpret_cast<uint32_t(*)[32]>(kk + 32));
      tmem_ld_32x32b_x32(tl + 64, *reinterpret_cast<uint32_t(*)[32]>(qk));
      tmem_ld_32x32b_x32(tl + 96, *reinterpret_cast<uint32_t(*)[32]>(qk + 32));
      tmem_wait_ld();
      const float gi = Gs[i], bi = Bs[i];
      float aq[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        const float e = j <= i ? __expf(gi - Gs[j]) : 0.f;
        Ls[i * LP + j] = j < i ? bi * e * __uint_as_float(kk[j]) : 0.f;
        aq[j] = j <= i ? a.scale * e * __uint_as_float(qk[j]) : 0.f;
      }
      uint4* dst = reinterpret_cast<uint4*>(a.Aqk + ((long)ch * C + i) * C);
#pragma unroll
      for (int m = 0; m < 8; ++m) dst[m] = pack8(aq + 8 * m);
      if (a.aux != nullptr) {
        float4* kr = reinterpret_cast<float4*>(a.aux + ((long)ch * 3 * C + i) * C);
        float4* qr = reinterpret_cast<float4*>(a.aux + ((long)ch * 3 * C + C + i) * C);
#pragma unroll
        for (int m = 0; m < 16; ++m) {
          kr[m] = make_float4(__uint_as_float(kk[4 * m]), __uint_as_float(kk[4 * m + 1]),
                              __uint_as_float(kk[4 * m + 2]), __uint_as_float(kk[4 * m + 3]));
          qr[m] = make_float4(a.scale * __uint_as_float(qk[4 * m]), a.scale * __uint_as_float(qk[4 * m + 1]),
                              a.scale * __uint_as_float(qk[4 * m + 2]), a.scale * __uint_as_float(qk[4 * m + 3]));
        }
      }
    }
  }
  ok = __syncthreads_and(ok);
  if (ok && tid < C) {
    // column j of T = (I + L)^-1 by forward substitution (four partial sums per row)
    const int j = tid;
    float x[C];
#pragma unroll
    for (int i = 0; i < C; ++i) {
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
      for (int l4 = 0; l4 < i / 4; ++l4) {
        const float4 lv = *reinterpret_cast<const float4*>(Ls + i * LP + 4 * l4);
        s0 = fmaf(lv.x, x[4 * l4], s0);
        s1 = fmaf(lv.y, x[4 * l4 + 1], s1);
        s2 = fmaf(lv.z, x[4 * l4 + 2], s2);
        s3 = fmaf(lv.w, x[4 * l4 + 3], s3);
      }
#pragma unroll
      for (int l = (i / 4) * 4; l < i; ++l) s0 = fmaf(Ls[i * LP + l], x[l], s0);
      x[i] = i < j ? 0.f : (i == j ? 1.f : -((s0 + s1) + (s2 + s3)));
    }
    if (a.aux != nullptr) {
      float* tcol = a.aux + ((long)ch * 3 * C + 2 * C) * C + j;
#pragma unroll
      for (int i = 0; i < C; ++i) tcol[i * C] = x[i];
    }
    const float sk = Bs[j] * __expf(Gs[j]), sv = Bs[j];
    const int cb = ((j >> 3)), cw = (j & 7) * 2;
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int off = i * 128 + (((cb ^ (i & 7))) << 4) + cw;
      *reinterpret_cast<__nv_bfloat16*>(sTk + off) = __float2bfloat16(x[i] * sk);
      *reinterpret_cast<__nv_bfloat16*>(sTv + off) = __float2bfloat16(x[i] * sv);
    }
  }
  fence_proxy_async();
  __syncthreads();
  if (ok && tid == 0) {
    tc_fence_after();
    const uint32_t tk = smem_u32(sTk), tv = smem_u32(sTv), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      umma_bf16_ss(tmem + 128, make_smem_desc_sw128(tk + k * 32, 16, 1024),
                   make_smem_desc_sw128(k_addr + k * 2048, BLK, 1024), make_idesc_bf16(128, 128, 0, 1), k > 0);
    const uint32_t idu = make_idesc_bf16(128, DV, 0, 1);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      umma_bf16_ss(tmem + 256, make_smem_desc_sw128(tv + k * 32, 16, 1024),
                   make_smem_desc_sw128(v_addr + k * 2048, BLK, 1024), idu, k > 0);
    umma_commit(mma2);
  }
  if (warp < 2) {
    const bool waited = __all_sync(0xffffffffu, ok && mbar_wait_bounded(mma2, 0, nullptr, a.status, kTimeoutEpilogue));
    if (waited) {
      tc_fence_after();
      const int i = tid;
      const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
      uint4* wd = reinterpret_cast<uint4*>(a.Wn + ((long)ch * C + i) * DK);
#pragma unroll 1
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tl + 128 + q4 * 32, r);
        tmem_wait_ld();
        float f[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) f[e] = -__uint_as_float(r[e]);
#pragma unroll
        for (int m = 0; m < 4; ++m) wd[q4 * 4 + m] = pack8(f + 8 * m);
      }
      uint4* ud = reinterpret_cast<uint4*>(a.U + ((long)ch * C + i) * DV);
#pragma unroll 1
      for (int q4 = 0; q4 < DV / 32; ++q4) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tl + 256 + q4 * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int m = 0; m < 4; ++m) ud[q4 * 4 + m] = pack8u(r + 8 * m);
      }
    }
  }
  if (tid < C) a.Gc[(long)ch * C + tid] = Gs[tid];
  if (tid == 0) {
    a.gam[ch] = __expf(GL);
    if (!ok) mbar_wait_bounded(full, 0, nullptr, nullptr, 0);  // no TMA copy may outlive the CTA
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TP_TMEM_COLS);
  }
}

// ============================================================================ state passes (tcgen05)
// warp 0 TMA, warp 1 MMA + TMEM owner, warps 2-9 the state lanes: warps w and w + 4 share TMEM lane
// quarter w % 4 and split its columns in halves (state columns, Delta columns, output tokens)
constexpr int ST_THREADS = 320;
constexpr int ST_LANE_THREADS = 256;
constexpr int VS = 128;          // value columns per CTA
constexpr int ST_OFF_WN = 0;
constexpr int ST_OFF_QG = 2 * BLK;
constexpr int ST_OFF_KD = 4 * BLK;
constexpr int ST_OFF_AQK = 6 * BLK;
constexpr int ST_OFF_X = 7 * BLK;  // U tile (forward) or dO tile (backward), 2 blocks of 64 value columns
constexpr int ST_STAGE = 9 * BLK;
constexpr int ST_STAGES = 2;
constexpr int ST_OFF_A1 = ST_STAGES * ST_STAGE;  // state^T in bf16: 128 rows x 128 cols, 2 blocks of 16 KB
constexpr int ST_OFF_A2 = ST_OFF_A1 + 2 * 128 * 128;  // (d)Delta^T in bf16: 128 rows x 64 cols
constexpr int ST_OFF_ID = ST_OFF_A2 + 128 * 128;  // forward: 64 x 64 identity (adds U^T to Delta^T on the MMA)
constexpr int ST_OFF_BAR = ST_OFF_ID + BLK;
constexpr int ST_SMEM = ST_OFF_BAR + 256 + 1024;
constexpr int ST_TMEM_COLS = 256;  // [0,128) state^T, [128,192) (d)Delta^T, [192,256) O^T

struct StateParams {
  const int* seq_chunks;   // [nseq + 1]
  const int* tok0;         // [Nc]
  const int* len;          // [Nc]
  const float* gam;        // [Nc, H]
  const float* S_in;       // fwd: initial state; bwd: gradient of the final state   [nseq, H, DK, DV] (nullable)
  float* S_out;            // fwd: final state;   bwd: gradient of the initial state [nseq, H, DK, DV] (nullable)
  __nv_bfloat16* states;   // fwd: S_c^T; bwd: G_{c+1}^T          [Nc, H, DV, DK] (fwd nullable)
  __nv_bfloat16* rows;     // fwd: Delta_c^T; bwd: dDelta_c^T     [Nc, H, DV, C]  (fwd nullable)
  __nv_bfloat16* out;      // fwd: o [T, H, DV] (nullable)
  int T;                   // rows of `out` (bounds of the debug build)
  int H, DV;
  int* status;
};

template <bool BWD>
__global__ void __launch_bounds__(ST_THREADS, 1)
    gdn_state_tc_kernel(const __grid_constant__ CUtensorMap mWn, const __grid_constant__ CUtensorMap mQg,
                        const __grid_constant__ CUtensorMap mKd, const __grid_constant__ CUtensorMap mAqk,
                        const __grid_constant__ CUtensorMap mX, StateParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + ST_OFF_BAR);
  uint64_t* full = bars;         // [2]
  uint64_t* empty = bars + 2;    // [2]
  uint64_t* a1_ready = bars + 4;
  uint64_t* d1_full = bars + 5;
  uint64_t* a2_ready = bars + 6;
  uint64_t* s_ready = bars + 7;
  uint64_t* o_empty = bars + 8;
  uint64_t* done = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 11);

  const int seq = blockIdx.x, h = blockIdx.y, v0 = blockIdx.z * VS;
  const int H = p.H, DV = p.DV;
  const int c_begin = p.seq_chunks[seq], c_end = p.seq_chunks[seq + 1];
  const int nch = c_end - c_begin;
  const bool want_out = BWD || p.out != nullptr;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(a1_ready, ST_LANE_THREADS);
    mbar_init(d1_full, 1);
    mbar_init(a2_ready, ST_LANE_THREADS);
    mbar_init(s_ready, 1);
    mbar_init(o_empty, ST_LANE_THREADS);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&mWn);
    tma_prefetch_desc(&mQg);
    tma_prefetch_desc(&mKd);
    tma_prefetch_desc(&mAqk);
    tma_prefetch_desc(&mX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, ST_TMEM_COLS);
    tmem_relinquish();
  }
  if (!BWD) {
    // 64 x 64 bf16 identity in the 128-byte-swizzled layout: B operand of Delta^T += U^T x I
    for (int i = threadIdx.x; i < 64 * 8; i += ST_THREADS) {
      const int r = i >> 3, cc = i & 7;
      uint4 z = make_uint4(0u, 0u, 0u, 0u);
      if ((r >> 3) == cc) reinterpret_cast<__nv_bfloat16*>(&z)[r & 7] = __float2bfloat16(1.f);
      *reinterpret_cast<uint4*>(smem + ST_OFF_ID + swz(r, cc)) = z;
    }
    fence_proxy_async();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0 && nch > 0) {
      int issued = 0;
      for (int j = 0; j < nch; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait_bounded(&empty[s], ((j >> 1) - 1) & 1, abort_flag, p.status, kTimeoutProducer))
          break;
        const int c = BWD ? c_end - 1 - j : c_begin + j;
        const int row = (c * H + h) * C;
        uint8_t* st = smem + s * ST_STAGE;
        mbar_arrive_expect_tx(&full[s], want_out ? 9 * BLK : 6 * BLK);
        tma_load_2d(st + ST_OFF_WN, &mWn, &full[s], 0, row);
        tma_load_2d(st + ST_OFF_WN + BLK, &mWn, &full[s], 64, row);
        tma_load_2d(st + ST_OFF_KD, &mKd, &full[s], 0, row);
        tma_load_2d(st + ST_OFF_KD + BLK, &mKd, &full[s], 64, row);
        if (BWD) {
          const int tr = p.tok0[c];
          tma_load_2d(st + ST_OFF_X, &mX, &full[s], h * DV + v0, tr);
          tma_load_2d(st + ST_OFF_X + BLK, &mX, &full[s], h * DV + v0 + 64, tr);
        } else {
          tma_load_2d(st + ST_OFF_X, &mX, &full[s], v0, row);
          tma_load_2d(st + ST_OFF_X + BLK, &mX, &full[s], v0 + 64, row);
        }
        if (want_out) {
          tma_load_2d(st + ST_OFF_QG, &mQg, &full[s], 0, row);
          tma_load_2d(st + ST_OFF_QG + BLK, &mQg, &full[s], 64, row);
          tma_load_2d(st + ST_OFF_AQK, &mAqk, &full[s], 0, row);
        }
        issued = j + 1;
      }
      // loads still in flight after an abort land before the CTA exits
      for (int j = issued > 2 ? issued - 2 : 0; j < issued; ++j)
        mbar_wait_bounded(&full[j & 1], (j >> 1) & 1, nullptr, nullptr, 0);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t id_n64 = make_idesc_bf16(128, 64, 0, 0);
      const uint32_t id_state = make_idesc_bf16(128, 128, 0, 1);
      const uint32_t id_do_aqk = make_idesc_bf16(128, 64, 1, 1);
      const uint32_t id_do_qg = make_idesc_bf16(128, 128, 1, 1);
      const uint32_t a1 = smem_u32(smem + ST_OFF_A1), a2 = smem_u32(smem + ST_OFF_A2);
      for (int j = 0; j < nch; ++j) {
        const int s = j & 1;
        const uint32_t st = smem_u32(smem + s * ST_STAGE);
        if (!mbar_wait_bounded(&full[s], (j >> 1) & 1, abort_flag, p.status, kTimeoutMma)) break;
        if (!mbar_wait_bounded(a1_ready, j & 1, abort_flag, p.status, kTimeoutMma)) break;
        tc_fence_after();
        // (d)Delta^T = state^T(bf16) x Wn^T (fwd) / Kd^T (bwd): K = dk, both K-major
        const uint32_t bsrc = st + (BWD ? ST_OFF_KD : ST_OFF_WN);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_bf16_ss(tmem + 128, make_smem_desc_sw128(a1 + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024),
                       make_smem_desc_sw128(bsrc + (k >> 2) * BLK + (k & 3) * 32, 16, 1024), id_n64, k > 0);
        {
          // bwd: += dO^T x Aqk; fwd: += U^T x I (Delta = U + Wn S exactly in fp32). K = chunk rows, A and B
          // MN-major
          const uint32_t bsum = BWD ? st + ST_OFF_AQK : smem_u32(smem + ST_OFF_ID);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_bf16_ss(tmem + 128, make_smem_desc_sw128(st + ST_OFF_X + k * 2048, BLK, 1024),
                         make_smem_desc_sw128(bsum + k * 2048, BLK, 1024), id_do_aqk, 1);
        }
        umma_commit(d1_full);
        if (BWD) {
          // G^T += dO^T x Qg (after the compute warps stored gamma * G^T)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_bf16_ss(tmem, make_smem_desc_sw128(st + ST_OFF_X + k * 2048, BLK, 1024),
                         make_smem_desc_sw128(st + ST_OFF_QG + k * 2048, BLK, 1024), id_do_qg, 1);
        } else if (want_out) {
          if (j > 0 && !mbar_wait_bounded(o_empty, (j - 1) & 1, abort_flag, p.status, kTimeoutMma)) break;
          tc_fence_after();
          // O^T = S^T x Qg^T
#pragma unroll
          for (int k = 0; k < 8; ++k)
            umma_bf16_ss(tmem + 192, make_smem_desc_sw128(a1 + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024),
                         make_smem_desc_sw128(st + ST_OFF_QG + (k >> 2) * BLK + (k & 3) * 32, 16, 1024), id_n64,
                         k > 0);
        }
        if (!mbar_wait_bounded(a2_ready, j & 1, abort_flag, p.status, kTimeoutMma)) break;
        tc_fence_after();
        // state^T += (d)Delta^T x Kd (fwd) / Wn (bwd): K = chunk rows, B MN-major
        const uint32_t bstate = st + (BWD ? ST_OFF_WN : ST_OFF_KD);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_bf16_ss(tmem, make_smem_desc_sw128(a2 + k * 32, 16, 1024),
                       make_smem_desc_sw128(bstate + k * 2048, BLK, 1024), id_state, 1);
        if (!BWD && want_out) {
          // O^T += Delta^T x Aqk^T
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_bf16_ss(tmem + 192, make_smem_desc_sw128(a2 + k * 32, 16, 1024),
                         make_smem_desc_sw128(st + ST_OFF_AQK + k * 32, 16, 1024), id_n64, 1);
        }
        umma_commit(s_ready);
        umma_commit(&empty[s]);
      }
      umma_commit(done);
      mbar_wait_bounded(done, 0, nullptr, nullptr, 0);
    }
  } else {
    // ---------------------------------------------------------------- state lanes
    // lane quarter = warp % 4 (the TMEM lanes this warp may access), half = which warp of the pair:
    // state columns [64 half, 64 half + 64), Delta columns and output tokens [32 half, 32 half + 32)
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int vl = quarter * 32 + lane;
    const int v = v0 + vl;
    const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16);
    uint8_t* A1 = smem + ST_OFF_A1;
    uint8_t* A2 = smem + ST_OFF_A2;
    const long sbase = ((long)seq * H + h) * DK * DV + v;

    auto drain_out = [&](int jj) {
      const int c = c_begin + jj;
      const int t0 = p.tok0[c] + 32 * half, n = p.len[c] - 32 * half;
      uint32_t r0[32];
      tmem_ld_32x32b_x32(tl + 192 + 32 * half, r0);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < n && PRISM_IN_BOUNDS(t0 + i, p.T, p.status))
          p.out[((long)(t0 + i) * H + h) * DV + v] = __float2bfloat16(__uint_as_float(r0[i]));
    };

#pragma unroll 1
    for (int q4 = 2 * half; q4 < 2 * half + 2; ++q4) {
      uint32_t r[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(p.S_in ? p.S_in[sbase + (long)(q4 * 32 + i) * DV] : 0.f);
      tmem_st_32x32b_x32(tl + q4 * 32, r);
    }
    tmem_wait_st();

    bool ok = nch > 0;
    for (int j = 0; j < nch; ++j) {
      const int c = BWD ? c_end - 1 - j : c_begin + j;
      const long ch = (long)c * H + h;
      if (j > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(s_ready, (j - 1) & 1, abort_flag, p.status,
                                                       kTimeoutEpilogue));
        if (!ok) break;
      }
      tc_fence_after();
      const float gm = p.gam[ch];
      {
        // both 32-column pieces of this half in flight before the first wait
        uint32_t r[2][32];
        tmem_ld_32x32b_x32(tl + 64 * half, r[0]);
        tmem_ld_32x32b_x32(tl + 64 * half + 32, r[1]);
        tmem_wait_ld();
        uint8_t* blk = A1 + half * 16384;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const uint4 pk = pack8u(r[e] + 8 * m);
            *reinterpret_cast<uint4*>(blk + swz(vl, e * 4 + m)) = pk;
            if (p.states != nullptr)
              reinterpret_cast<uint4*>(p.states + (ch * DV + v) * DK + (2 * half + e) * 32)[m] = pk;
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) r[e][i] = __float_as_uint(__uint_as_float(r[e][i]) * gm);
        }
        tmem_st_32x32b_x32(tl + 64 * half, r[0]);
        tmem_st_32x32b_x32(tl + 64 * half + 32, r[1]);
      }
      tmem_wait_st();
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(a1_ready);
      if (!BWD && want_out && j > 0) {
        drain_out(j - 1);
        tc_fence_before();
        mbar_arrive(o_empty);
      }
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(d1_full, j & 1, abort_flag, p.status, kTimeoutEpilogue));
      if (!ok) break;
      tc_fence_after();
      uint32_t r0[32];
      tmem_ld_32x32b_x32(tl + 128 + 32 * half, r0);
      tmem_wait_ld();
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const uint4 pk = pack8u(r0 + 8 * m);
        *reinterpret_cast<uint4*>(A2 + swz(vl, 4 * half + m)) = pk;
        if (p.rows != nullptr) reinterpret_cast<uint4*>(p.rows + (ch * DV + v) * C)[4 * half + m] = pk;
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(a2_ready);
    }
    if (nch == 0 && p.S_out != nullptr) {
      // an empty sequence leaves its state unchanged
      for (int d = 64 * half; d < 64 * half + 64; ++d)
        p.S_out[sbase + (long)d * DV] = p.S_in ? p.S_in[sbase + (long)d * DV] : 0.f;
    }
    if (ok) {
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(s_ready, (nch - 1) & 1, abort_flag, p.status,
                                                     kTimeoutEpilogue));
      if (ok) {
        tc_fence_after();
        if (!BWD && want_out) drain_out(nch - 1);
        if (p.S_out != nullptr) {
#pragma unroll 1
          for (int q4 = 2 * half; q4 < 2 * half + 2; ++q4) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tl + q4 * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) p.S_out[sbase + (long)(q4 * 32 + i) * DV] = __uint_as_float(r[i]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, ST_TMEM_COLS);
  }
}

// ============================================================================ dv contractions (tcgen05)
constexpr int DV_THREADS = 128;
constexpr int DV_TMEM_COLS = 512;

struct DvParams {
  const int* tok0;
  float* dWnT;   // [Nc, H, DK, C]   dWn^T
  float* dQgT;   // [Nc, H, DK, C]   dQg^T
  float* dKdT;   // [Nc, H, DK, C]   dKd^T
  float* dAqk;   // [Nc, H, C, C]
  float* dDV;    // [Nc, H, C, C]    dDelta V^T (nullable: not computed)
  float* dgam;   // [Nc, H]
  int H, DV;
  int* status;
  int accumulate;  // add to the outputs instead of writing them (a second state pass over the same chunks)
};

// 16 fp32 values of one TMEM row half (r0: columns 0..31 of the pair, r1: 32..63) into dst[0..16)
PRISM_DEVICE void put_row64(float4* dst, const uint32_t* r0, const uint32_t* r1, bool acc) {
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    float4 a = make_float4(__uint_as_float(r0[4 * m]), __uint_as_float(r0[4 * m + 1]),
                           __uint_as_float(r0[4 * m + 2]), __uint_as_float(r0[4 * m + 3]));
    float4 b = make_float4(__uint_as_float(r1[4 * m]), __uint_as_float(r1[4 * m + 1]),
                           __uint_as_float(r1[4 * m + 2]), __uint_as_float(r1[4 * m + 3]));
    if (acc) {
      const float4 x = dst[m], y = dst[m + 8];
      a = make_float4(a.x + x.x, a.y + x.y, a.z + x.z, a.w + x.w);
      b = make_float4(b.x + y.x, b.y + y.y, b.z + y.z, b.w + y.w);
    }
    dst[m] = a;
    dst[m + 8] = b;
  }
}

// Tile order in shared memory (bytes, DV = value width):
//   S^T [DV x DK] | G^T [DV x DK] | dO [C x DV] | dDelta^T [DV x C] | Delta^T [DV x C]
// The padded M = 128 products read 64 rows past the dO and dDelta^T tiles; those
// rows are the next tile (never past the end of the allocation) and land in TMEM
// lanes 64..127, which are not read.
__global__ void __launch_bounds__(DV_THREADS, 1)
    gdn_bwd_dv_kernel(const __grid_constant__ CUtensorMap mS, const __grid_constant__ CUtensorMap mG,
                      const __grid_constant__ CUtensorMap mDO, const __grid_constant__ CUtensorMap mDD,
                      const __grid_constant__ CUtensorMap mDL, const __grid_constant__ CUtensorMap mV,
                      DvParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int DV = p.DV, H = p.H;
  const int OFF_S = 0, OFF_GN = DV * 256, OFF_DO = DV * 512, OFF_DD = DV * 640, OFF_DL = DV * 768;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + DV * 896);
  uint64_t* full_a = bars;
  uint64_t* full_b = bars + 1;
  uint64_t* mma_a = bars + 2;
  uint64_t* mma_b = bars + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  float* red = reinterpret_cast<float*>(bars + 5);  // [4]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long ch = blockIdx.x;
  const int c = (int)(ch / H), h = (int)(ch % H);

  if (threadIdx.x == 0) {
    mbar_init(full_a, 1);
    mbar_init(full_b, 1);
    mbar_init(mma_a, 1);
    mbar_init(mma_b, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, DV_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nb = DV / 64;

  if (threadIdx.x == 0) {
    const int tr = p.tok0[c];
    mbar_arrive_expect_tx(full_a, DV * 896);
    for (int rb = 0; rb < nb; ++rb) {
      const int row = (int)(ch * DV) + rb * 64;
      for (int cb = 0; cb < 2; ++cb) {
        tma_load_2d(smem + OFF_S + cb * DV * 128 + rb * BLK, &mS, full_a, cb * 64, row);
        tma_load_2d(smem + OFF_GN + cb * DV * 128 + rb * BLK, &mG, full_a, cb * 64, row);
      }
      tma_load_2d(smem + OFF_DD + rb * BLK, &mDD, full_a, 0, row);
      tma_load_2d(smem + OFF_DL + rb * BLK, &mDL, full_a, 0, row);
      tma_load_2d(smem + OFF_DO + rb * BLK, &mDO, full_a, h * DV + rb * 64, tr);
    }
    bool b_issued = false;
    bool ok = mbar_wait_bounded(full_a, 0, nullptr, p.status, kTimeoutMma);
    if (ok) {
      tc_fence_after();
      const uint32_t sS = smem_u32(smem + OFF_S), sG = smem_u32(smem + OFF_GN), sO = smem_u32(smem + OFF_DO);
      const uint32_t sD = smem_u32(smem + OFF_DD), sL = smem_u32(smem + OFF_DL);
      const uint32_t lbo = DV * 128;
      const int ks = DV / 16;
      for (int k = 0; k < ks; ++k) {
        const uint64_t aS = make_smem_desc_sw128(sS + k * 2048, lbo, 1024);
        const uint64_t aG = make_smem_desc_sw128(sG + k * 2048, lbo, 1024);
        const uint64_t kO = make_smem_desc_sw128(sO + (k >> 2) * BLK + (k & 3) * 32, 16, 1024);
        const uint64_t mD = make_smem_desc_sw128(sD + k * 2048, lbo, 1024);
        const uint64_t mL = make_smem_desc_sw128(sL + k * 2048, lbo, 1024);
        const uint32_t acc = k > 0;
        umma_bf16_ss(tmem + 0, aS, mD, make_idesc_bf16(128, 64, 1, 1), acc);     // dWn^T = S dDelta^T
        umma_bf16_ss(tmem + 64, aS, kO, make_idesc_bf16(128, 64, 1, 0), acc);    // dQg^T = S dO^T
        umma_bf16_ss(tmem + 128, kO, mL, make_idesc_bf16(128, 64, 0, 1), acc);   // dAqk = dO Delta^T
        umma_bf16_ss(tmem + 192, aG, mL, make_idesc_bf16(128, 64, 1, 1), acc);   // dKd^T = G Delta^T
        umma_bf16_ss(tmem + 256, aS, aG, make_idesc_bf16(128, 128, 1, 1), acc);  // S G^T (trace = dgamma)
      }
      umma_commit(mma_a);
      ok = mbar_wait_bounded(mma_a, 0, nullptr, p.status, kTimeoutMma);
      if (ok && p.dDV != nullptr) {
        // the value tile replaces dO
        mbar_arrive_expect_tx(full_b, DV * 128);
        for (int rb = 0; rb < nb; ++rb) tma_load_2d(smem + OFF_DO + rb * BLK, &mV, full_b, h * DV + rb * 64, tr);
        b_issued = true;
        ok = mbar_wait_bounded(full_b, 0, nullptr, p.status, kTimeoutMma);
        if (ok) {
          tc_fence_after();
          for (int k = 0; k < ks; ++k) {
            const uint64_t mD = make_smem_desc_sw128(sD + k * 2048, lbo, 1024);
            const uint64_t kV = make_smem_desc_sw128(sO + (k >> 2) * BLK + (k & 3) * 32, 16, 1024);
            umma_bf16_ss(tmem + 384, mD, kV, make_idesc_bf16(128, 64, 1, 0), k > 0);  // dDelta V^T
          }
          umma_commit(mma_b);
          mbar_wait_bounded(mma_b, 0, nullptr, p.status, kTimeoutMma);
        }
      }
    }
    if (!ok) {
      // make sure no TMA copy is still writing shared memory
      mbar_wait_bounded(full_a, 0, nullptr, nullptr, 0);
      if (b_issued) mbar_wait_bounded(full_b, 0, nullptr, nullptr, 0);
    }
  }
  __syncwarp();
  // ---------------------------------------------------------------- epilogue: lane = row
  const bool ok_a = __all_sync(0xffffffffu, mbar_wait_bounded(mma_a, 0, nullptr, p.status, kTimeoutEpilogue));
  const int r = warp * 32 + lane;
  const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
  float gsum = 0.f;
  if (ok_a) {
    tc_fence_after();
    float* outs[3] = {p.dWnT, p.dQgT, p.dKdT};
    const int cols[3] = {0, 64, 192};
#pragma unroll 1
    for (int o = 0; o < 3; ++o) {
      uint32_t r0[32], r1[32];
      tmem_ld_32x32b_x32(tl + cols[o], r0);
      tmem_ld_32x32b_x32(tl + cols[o] + 32, r1);
      tmem_wait_ld();
      put_row64(reinterpret_cast<float4*>(outs[o] + (ch * DK + r) * C), r0, r1, p.accumulate);
    }
    if (warp < 2) {
      uint32_t r0[32], r1[32];
      tmem_ld_32x32b_x32(tl + 128, r0);
      tmem_ld_32x32b_x32(tl + 160, r1);
      tmem_wait_ld();
      put_row64(reinterpret_cast<float4*>(p.dAqk + (ch * C + r) * C), r0, r1, p.accumulate);
    }
    {
      // diagonal element (r, r) of S G^T: columns 256 + 32 * warp .. + 31 hold it at index lane
      uint32_t rg[32];
      tmem_ld_32x32b_x32(tl + 256 + 32 * warp, rg);
      tmem_wait_ld();
      float dval = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) dval = (i == lane) ? __uint_as_float(rg[i]) : dval;
      gsum = warp_sum(dval);
    }
  }
  if (lane == 0) red[warp] = gsum;
  const bool ok_b = ok_a && p.dDV != nullptr &&
                    __all_sync(0xffffffffu, mbar_wait_bounded(mma_b, 0, nullptr, p.status, kTimeoutEpilogue));
  if (ok_b && warp < 2) {
    tc_fence_after();
    uint32_t r0[32], r1[32];
    tmem_ld_32x32b_x32(tl + 384, r0);
    tmem_ld_32x32b_x32(tl + 416, r1);
    tmem_wait_ld();
    put_row64(reinterpret_cast<float4*>(p.dDV + (ch * C + r) * C), r0, r1, p.accumulate);
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) p.dgam[ch] = (p.accumulate ? p.dgam[ch] : 0.f) + red[0] + red[1] + red[2] + red[3];
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, DV_TMEM_COLS);
  }
}

// ============================================================================ chunk-local backward
constexpr int LB_THREADS = 256;
constexpr int P65 = 65;
constexpr int LB_SMEM = (3 * C * KP + 6 * C * P65 + 4 * C) * 4;

struct LocalArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const float* g;
  const float* beta;
  const int* tok0;
  const int* len;
  const float* Gc;      // [Nc, H, C]
  const float* aux;     // [Nc * H, 3, C, C]: k.k, s q.k, T (from the prep recompute)
  const float* dWnT;    // [Nc, H, DK, C]
  const float* dQgT;
  const float* dKdT;
  const float* dAqk;    // [Nc, H, C, C]
  const float* dDV;     // [Nc, H, C, C]
  const float* dgam;    // [Nc, H]
  const __nv_bfloat16* dDT;  // [Nc, H, DV, C]
  __nv_bfloat16* dq;    // [T, H, DK]
  __nv_bfloat16* dk;    // [T, H, DK]
  __nv_bfloat16* dv;    // [T, H, DV]
  float* dg;            // [T, H]
  float* dbeta;         // [T, H]
  float scale;
  int H, DV;
};

// Sum over the 16 lanes that share a row (lanes tj = 0..15 of one half warp).
PRISM_DEVICE float half_warp_sum(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(LB_THREADS, 1) gdn_bwd_local_kernel(LocalArgs a) {
  extern __shared__ float sm[];
  float* ks = sm;                 // k rows
  float* qs = ks + C * KP;        // s q rows
  float* ws = qs + C * KP;        // transposed loads of dWn / dQg / dKd
  float* Ts = ws + C * KP;        // T = (I + L)^-1
  float* KK = Ts + C * P65;       // k_i . k_j
  float* QK = KK + C * P65;       // s q_i . k_j
  float* X1 = QK + C * P65;
  float* X2 = X1 + C * P65;
  float* X3 = X2 + C * P65;
  float* Gs = X3 + C * P65;
  float* Bs = Gs + C;
  float* dG = Bs + C;
  float* dB = dG + C;
  const int H = a.H, DV = a.DV;
  const long ch = blockIdx.x;
  const int c = (int)(ch / H), h = (int)(ch % H);
  const int t0 = a.tok0[c], n = a.len[c];
  const int tid = threadIdx.x;
  const int ti = tid >> 4, tj = tid & 15;

  if (tid < C) {
    dG[tid] = 0.f;
    dB[tid] = 0.f;
  }
  load_chunk_kq(a.q, a.k, a.g, a.beta, t0, n, h, H, a.scale, ks, qs, Gs, Bs);
  {
    // k.k, s q.k and T = (I + L)^-1 come from the prep recompute
    const float* src = a.aux + ch * 3 * C * C;
    for (int e = tid; e < C * C; e += LB_THREADS) {
      const int i = e / C, j = e % C;
      KK[i * P65 + j] = src[e];
      QK[i * P65 + j] = src[C * C + e];
      Ts[i * P65 + j] = src[2 * C * C + e];
    }
  }
  // dW = -dWn, stored [i][a]
  for (int e = tid; e < DK * C; e += LB_THREADS) {
    const int aa = e / C, i = e % C;
    ws[i * KP + aa] = -a.dWnT[(ch * DK + aa) * C + i];
  }
  __syncthreads();

  float dkr[4][8], dqr[4][8];
  // dBk = T^T dW; dk += beta e^G dBk; dbeta, dG from Bk = beta e^G k
  {
    float acc[4][8];
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int y = 0; y < 8; ++y) acc[x][y] = 0.f;
#pragma unroll 4
    for (int l = 0; l < C; ++l) {
      float t[4], w[8];
#pragma unroll
      for (int x = 0; x < 4; ++x) t[x] = Ts[l * P65 + ti + 16 * x];
#pragma unroll
      for (int y = 0; y < 8; ++y) w[y] = ws[l * KP + tj + 16 * y];
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 8; ++y) acc[x][y] = fmaf(t[x], w[y], acc[x][y]);
    }
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      const int i = ti + 16 * x;
      const float eg = __expf(Gs[i]);
      float part = 0.f;
#pragma unroll
      for (int y = 0; y < 8; ++y) {
        dkr[x][y] = Bs[i] * eg * acc[x][y];
        part = fmaf(acc[x][y], ks[i * KP + tj + 16 * y], part);
      }
      part = half_warp_sum(part);
      if (tj == 0) {
        atomicAdd(&dB[i], eg * part);
        atomicAdd(&dG[i], Bs[i] * eg * part);
      }
    }
  }
  // dT = dW Bk^T + beta_j dDelta V^T  ->  X2
  {
    float acc[4][4];
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) acc[x][y] = 0.f;
#pragma unroll 4
    for (int d = 0; d < DK; ++d) {
      float u[4], w[4];
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        u[x] = ws[(ti + 16 * x) * KP + d];
        w[x] = ks[(tj + 16 * x) * KP + d];
      }
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(u[x], w[y], acc[x][y]);
    }
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) {
        const int i = ti + 16 * x, j = tj + 16 * y;
        X2[i * P65 + j] = Bs[j] * (__expf(Gs[j]) * acc[x][y] + a.dDV[(ch * C + i) * C + j]);
      }
  }
  __syncthreads();
  // Z = T^T dT -> X3
  {
    float acc[4][4];
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) acc[x][y] = 0.f;
#pragma unroll 4
    for (int l = 0; l < C; ++l) {
      float u[4], w[4];
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        u[x] = Ts[l * P65 + ti + 16 * x];
        w[x] = X2[l * P65 + tj + 16 * x];
      }
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(u[x], w[y], acc[x][y]);
    }
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) X3[(ti + 16 * x) * P65 + tj + 16 * y] = acc[x][y];
  }
  __syncthreads();
  // dL = -Z T^T (strictly lower) -> X2
  {
    float acc[4][4];
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) acc[x][y] = 0.f;
#pragma unroll 4
    for (int m = 0; m < C; ++m) {
      float u[4], w[4];
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        u[x] = X3[(ti + 16 * x) * P65 + m];
        w[x] = Ts[(tj + 16 * x) * P65 + m];
      }
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(u[x], w[y], acc[x][y]);
    }
    __syncthreads();
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) {
        const int i = ti + 16 * x, j = tj + 16 * y;
        X2[i * P65 + j] = j < i ? -acc[x][y] : 0.f;
      }
  }
  __syncthreads();
  // L terms (-> dKK in X1) and Aqk terms (-> dA in X3)
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const int i = ti + 16 * x;
    float rb = 0.f, rg = 0.f;
#pragma unroll
    for (int y = 0; y < 4; ++y) {
      const int j = tj + 16 * y;
      const float e = j <= i ? __expf(Gs[i] - Gs[j]) : 0.f;
      const float dl = X2[i * P65 + j];
      const float kk = KK[i * P65 + j];
      const float m = dl * Bs[i] * e * kk;
      rb = fmaf(dl * e, kk, rb);
      rg += m;
      if (j < i) atomicAdd(&dG[j], -m);
      X1[i * P65 + j] = dl * Bs[i] * e;
      const float daq = j <= i ? a.dAqk[(ch * C + i) * C + j] : 0.f;
      const float pq = daq * QK[i * P65 + j] * e;
      rg += pq;
      if (j <= i) atomicAdd(&dG[j], -pq);
      X3[i * P65 + j] = daq * e;
    }
    rb = half_warp_sum(rb);
    rg = half_warp_sum(rg);
    if (tj == 0) {
      atomicAdd(&dB[i], rb);
      atomicAdd(&dG[i], rg);
    }
  }
  __syncthreads();
  // X2 = dKK + dKK^T
#pragma unroll
  for (int x = 0; x < 4; ++x)
#pragma unroll
    for (int y = 0; y < 4; ++y) {
      const int i = ti + 16 * x, j = tj + 16 * y;
      X2[i * P65 + j] = X1[i * P65 + j] + X1[j * P65 + i];
    }
  __syncthreads();
  // dk += (dKK + dKK^T) k + dA^T (s q);  dq = s dA k
  {
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int y = 0; y < 8; ++y) dqr[x][y] = 0.f;
#pragma unroll 2
    for (int j = 0; j < C; ++j) {
      float c1[4], da[4], dat[4], kj[8], qj[8];
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        const int i = ti + 16 * x;
        c1[x] = X2[i * P65 + j];
        da[x] = X3[i * P65 + j];
        dat[x] = X3[j * P65 + i];
      }
#pragma unroll
      for (int y = 0; y < 8; ++y) {
        kj[y] = ks[j * KP + tj + 16 * y];
        qj[y] = qs[j * KP + tj + 16 * y];
      }
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 8; ++y) {
          dkr[x][y] = fmaf(c1[x], kj[y], dkr[x][y]);
          dkr[x][y] = fmaf(dat[x], qj[y], dkr[x][y]);
          dqr[x][y] = fmaf(da[x], kj[y], dqr[x][y]);
        }
    }
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int y = 0; y < 8; ++y) dqr[x][y] *= a.scale;
  }
  __syncthreads();
  // dQg: dq += s e^G dQg; dG += dQg . Qg
  for (int e = tid; e < DK * C; e += LB_THREADS) {
    const int aa = e / C, i = e % C;
    ws[i * KP + aa] = a.dQgT[(ch * DK + aa) * C + i];
  }
  __syncthreads();
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const int i = ti + 16 * x;
    const float eg = __expf(Gs[i]);
    float part = 0.f;
#pragma unroll
    for (int y = 0; y < 8; ++y) {
      const float w = ws[i * KP + tj + 16 * y];
      dqr[x][y] = fmaf(a.scale * eg, w, dqr[x][y]);
      part = fmaf(w, qs[i * KP + tj + 16 * y], part);
    }
    part = half_warp_sum(part);
    if (tj == 0) atomicAdd(&dG[i], eg * part);
  }
  __syncthreads();
  // dKd: dk += e^(G_L - G) dKd; dG_i -= r_i; dG_L += r_i
  for (int e = tid; e < DK * C; e += LB_THREADS) {
    const int aa = e / C, i = e % C;
    ws[i * KP + aa] = a.dKdT[(ch * DK + aa) * C + i];
  }
  __syncthreads();
  {
    const float GL = Gs[C - 1];
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      const int i = ti + 16 * x;
      const float ed = __expf(GL - Gs[i]);
      float part = 0.f;
#pragma unroll
      for (int y = 0; y < 8; ++y) {
        const float w = ws[i * KP + tj + 16 * y];
        dkr[x][y] = fmaf(ed, w, dkr[x][y]);
        part = fmaf(w, ks[i * KP + tj + 16 * y], part);
      }
      part = half_warp_sum(part) * ed;
      if (tj == 0) {
        atomicAdd(&dG[i], -part);
        atomicAdd(&dG[C - 1], part);
      }
    }
    if (tid == 0) atomicAdd(&dG[C - 1], __expf(GL) * a.dgam[ch]);
  }
  // dv = beta T^T dDelta; dbeta += dBv . v
  for (int col = tid; col < DV; col += LB_THREADS) {
    float d[C];
    const uint4* src = reinterpret_cast<const uint4*>(a.dDT + (ch * DV + col) * C);
#pragma unroll
    for (int m = 0; m < 8; ++m) unpack8(src[m], d + 8 * m);
    const __nv_bfloat16* vp = a.v + (long)h * DV + col;
    __nv_bfloat16* dvp = a.dv + (long)h * DV + col;
#pragma unroll
    for (int i = 0; i < C; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int l = i; l < C; ++l) acc = fmaf(Ts[l * P65 + i], d[l], acc);
      float contrib = 0.f;
      if (i < n) {
        dvp[(long)(t0 + i) * H * DV] = __float2bfloat16(Bs[i] * acc);
        contrib = acc * bf2f(vp[(long)(t0 + i) * H * DV]);
      }
      contrib = warp_sum(contrib);
      if ((tid & 31) == 0) atomicAdd(&dB[i], contrib);
    }
  }
  __syncthreads();
  // dg = reverse cumulative sum of dG; write dq, dk, dg, dbeta
  if (tid < 32) {
    float x0 = dG[tid], x1 = dG[tid + 32];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y0 = __shfl_down_sync(0xffffffffu, x0, o);
      const float y1 = __shfl_down_sync(0xffffffffu, x1, o);
      if (tid + o < 32) {
        x0 += y0;
        x1 += y1;
      }
    }
    x0 += __shfl_sync(0xffffffffu, x1, 0);
    if (tid < n) {
      a.dg[(long)(t0 + tid) * H + h] = x0;
      a.dbeta[(long)(t0 + tid) * H + h] = dB[tid];
    }
    if (tid + 32 < n) {
      a.dg[(long)(t0 + tid + 32) * H + h] = x1;
      a.dbeta[(long)(t0 + tid + 32) * H + h] = dB[tid + 32];
    }
  }
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const int i = ti + 16 * x;
    if (i < n) {
      const long off = ((long)(t0 + i) * H + h) * DK;
#pragma unroll
      for (int y = 0; y < 8; ++y) {
        a.dq[off + tj + 16 * y] = __float2bfloat16(dqr[x][y]);
        a.dk[off + tj + 16 * y] = __float2bfloat16(dkr[x][y]);
      }
    }
  }
}

// ============================================================================ chunk-local backward (tcgen05)
// Same WY / decay backward as gdn_bwd_local_kernel, with every product on the tensor cores.
// One CTA (4 warps) per (chunk, head); warps 0-1 own the chunk's 64 rows (TMEM lanes 0..63,
// one row per thread) for every epilogue, all warps stage operands. With T = (I + L)^-1 and
// dW = -dWn, the products are (each M = 128 with rows 64..127 of the A operand reading the
// next tile into TMEM lanes that are never read):
//   D1 = T^T dW                 [i, a]   -> dBk; dk starts as beta e^G D1 (stored back)
//   D2 = dW k^T                 [i, j]   -> X2 = beta_j (e^G_j D2 + dDelta V^T)
//   D3 = T^T X2                 [i, m]   -> Z
//   D4 = Z T^T                  [i, j]   -> dL = -D4 (strictly lower), X1, X3 = s dAqk o E
//   D5 = dk + (X1 + X1^T) k + X3^T q     -> dk (plus e^(G_L - G) dKd)
//   D6 = X3 k                   [i, a]   -> dq (plus s e^G dQg)
//   D7 = T^T dDelta             [i, col] -> dv = beta D7
// Operands are bf16 in 128-byte-swizzled shared memory; accumulation is fp32 in TMEM.
namespace lt {
constexpr int THREADS = 128;
// 256 TMEM columns and under 100 KB of shared memory per CTA, so two CTAs share an SM and
// one CTA's loads and epilogues hide the other's MMA and barrier latency:
//   TMEM: D1/D5 [0,128), D2 [128,192), D3 [192,256), D4 [128,192), D6 [128,256), D7 [0,DV)
//   smem blocks (8 KB each): K 0-1, Q 2-3, T 4, dW 5-6, X2 7, Z 8, X1+X1^T 9, s X3 10, slack 11
//   (read as the unused rows 64..127 of M = 128 operands). Blocks 5-8 are reused: fp32 X1 and
//   the dG column terms while the dL epilogue runs, then dDelta^T for D7.
constexpr int TMEM_COLS = 256;
constexpr int OFF_K = 0, OFF_Q = 2 * BLK, OFF_T = 4 * BLK, OFF_W = 5 * BLK, OFF_X2 = 7 * BLK, OFF_Z = 8 * BLK;
constexpr int OFF_XS = 9 * BLK, OFF_X3 = 10 * BLK, OFF_DD = OFF_W, OFF_F = OFF_W, OFF_END = 12 * BLK;
constexpr int FT = C * C;  // one fp32 64 x 64 tile (rows skewed: element (r, j) at r * 64 + ((j + r) & 63))
constexpr int SMEM = OFF_END + 4 * C * 4 + 64 + 1024;

// fp32 tile element (r, j) with the row skew that keeps row-per-thread and column-per-thread
// accesses free of bank conflicts
PRISM_DEVICE int sk(int r, int j) { return r * 64 + ((j + r) & 63); }

// Writes 8 consecutive bf16 (columns 8cc..8cc+7) of row r into a swizzled tile of 64-column blocks.
PRISM_DEVICE void put8(uint8_t* tile, int r, int cc, uint4 v) {
  *reinterpret_cast<uint4*>(tile + (cc >> 3) * BLK + swz(r, cc & 7)) = v;
}

PRISM_DEVICE void get_row_f(const uint8_t* tile, int r, int cc, float* f) {
  unpack8(*reinterpret_cast<const uint4*>(tile + (cc >> 3) * BLK + swz(r, cc & 7)), f);
}

PRISM_DEVICE uint64_t kmaj(uint32_t base, int k) { return make_smem_desc_sw128(base + (k >> 2) * BLK + (k & 3) * 32, 16, 1024); }
PRISM_DEVICE uint64_t mnmaj(uint32_t base, int k) { return make_smem_desc_sw128(base + k * 2048, BLK, 1024); }

PRISM_DEVICE void ld32(uint32_t taddr, float* f) {
  uint32_t r[32];
  tmem_ld_32x32b_x32(taddr, r);
  tmem_wait_ld();
#pragma unroll
  for (int e = 0; e < 32; ++e) f[e] = __uint_as_float(r[e]);
}
}  // namespace lt

struct LocalTcArgs {
  LocalArgs a;
  int* status;
};

__global__ void __launch_bounds__(lt::THREADS, 1)
    gdn_bwd_local_tc_kernel(const __grid_constant__ CUtensorMap mQ, const __grid_constant__ CUtensorMap mK,
                            const __grid_constant__ CUtensorMap mDD, LocalTcArgs args) {
  using namespace lt;
  const LocalArgs& a = args.a;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t *sK = smem + OFF_K, *sQ = smem + OFF_Q, *sT = smem + OFF_T, *sW = smem + OFF_W;
  uint8_t *sX2 = smem + OFF_X2, *sZ = smem + OFF_Z, *sXS = smem + OFF_XS, *sX3 = smem + OFF_X3;
  uint8_t* sDD = smem + OFF_DD;
  float* X1s = reinterpret_cast<float*>(smem + OFF_F);
  float* Mc = X1s + FT;   // -(dG contributions) per (row, column): summed over rows by warps 2-3
  float* Gs = reinterpret_cast<float*>(smem + OFF_END);
  float* Bs = Gs + C;
  float* dGc = Bs + C;
  float* misc = dGc + C;  // [0]: dG of the last row from the dKd terms
  uint64_t* bars = reinterpret_cast<uint64_t*>(misc + C);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7);
  const int H = a.H, DV = a.DV, nvb = DV / 64;
  const long ch = blockIdx.x;
  const int c = (int)(ch / H), h = (int)(ch % H);
  const int t0 = a.tok0[c], n = a.len[c];
  const int tid = threadIdx.x, warp = tid >> 5;
  const bool owner = warp < 2;  // threads 0..63: one chunk row each (TMEM lanes 0..63)
  const int i = tid;

  if (tid == 0) {
#pragma unroll
    for (int b = 0; b < 7; ++b) mbar_init(&bars[b], 1);
    misc[0] = 0.f;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (tid == 0) {
    mbar_arrive_expect_tx(&bars[0], 4 * BLK);
    tma_load_2d(sK, &mK, &bars[0], h * DK, t0);
    tma_load_2d(sK + BLK, &mK, &bars[0], h * DK + 64, t0);
    tma_load_2d(sQ, &mQ, &bars[0], h * DK, t0);
    tma_load_2d(sQ + BLK, &mQ, &bars[0], h * DK + 64, t0);
  }
  if (warp == 0) {
    const int l = tid;
    float x0 = l < n ? a.g[(long)(t0 + l) * H + h] : 0.f;
    float x1 = l + 32 < n ? a.g[(long)(t0 + l + 32) * H + h] : 0.f;
    Bs[l] = l < n ? a.beta[(long)(t0 + l) * H + h] : 0.f;
    Bs[l + 32] = l + 32 < n ? a.beta[(long)(t0 + l + 32) * H + h] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y0 = __shfl_up_sync(0xffffffffu, x0, o);
      const float y1 = __shfl_up_sync(0xffffffffu, x1, o);
      if (l >= o) {
        x0 += y0;
        x1 += y1;
      }
    }
    x1 += __shfl_sync(0xffffffffu, x0, 31);
    Gs[l] = x0;
    Gs[l + 32] = x1;
  }
  // operands staged by all threads: T (rows l, cols i) and dW = -dWn (rows i, cols a); the loops
  // are unrolled so that each thread's global loads are in flight together
  const float* aux = a.aux + ch * 3 * C * C;
#pragma unroll 4
  for (int e = tid; e < C * 8; e += THREADS) {
    const int l = e >> 3, cc = e & 7;
    const float4 x = reinterpret_cast<const float4*>(aux + 2 * C * C + l * C)[2 * cc];
    const float4 y = reinterpret_cast<const float4*>(aux + 2 * C * C + l * C)[2 * cc + 1];
    const float f[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
    put8(sT, l, cc, pack8(f));
  }
#pragma unroll 8
  for (int e = tid; e < C * 16; e += THREADS) {
    const int r = e & 63, a8 = (e >> 6) * 8;
    float f[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) f[m] = -a.dWnT[(ch * DK + a8 + m) * C + r];
    put8(sW, r, a8 >> 3, pack8(f));
  }
  bool ok = __syncthreads_and(mbar_wait_bounded(&bars[0], 0, nullptr, args.status, kTimeoutProducer));
  if (ok && n < C) {
    // rows past the end of the sequence hold the next sequence's tokens: zero them
    const int per = (C - n) * 8;
    for (int e = tid; e < 4 * per; e += THREADS) {
      const int b = e / per, rem = e % per;
      *reinterpret_cast<uint4*>(smem + b * BLK + swz(n + rem / 8, rem % 8)) = make_uint4(0, 0, 0, 0);
    }
  }
  fence_proxy_async();
  ok = __syncthreads_and(ok);

  const uint32_t aK = smem_u32(sK), aQ = smem_u32(sQ), aT = smem_u32(sT), aW = smem_u32(sW);
  const uint32_t aX2 = smem_u32(sX2), aZ = smem_u32(sZ), aXS = smem_u32(sXS), aX3 = smem_u32(sX3);
  const uint32_t aDD = smem_u32(sDD);
  const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  const float Gi = Gs[i & 63], Bi = Bs[i & 63], egi = __expf(Gi), GL = Gs[C - 1];
  float dB_own = 0.f, dG_own = 0.f;

  // ---- D1 = T^T dW, D2 = dW k^T
  if (ok && tid == 0) {
    tc_fence_after();
#pragma unroll
    for (int k = 0; k < 4; ++k) umma_bf16_ss(tmem, mnmaj(aT, k), mnmaj(aW, k), make_idesc_bf16(128, 128, 1, 1), k > 0);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      umma_bf16_ss(tmem + 128, kmaj(aW, k), kmaj(aK, k), make_idesc_bf16(128, 64, 0, 0), k > 0);
    umma_commit(&bars[1]);
  }
  if (owner) {
    ok = __all_sync(0xffffffffu, ok && mbar_wait_bounded(&bars[1], 0, nullptr, args.status, kTimeoutEpilogue));
    if (ok) {
      tc_fence_after();
      float part = 0.f;
#pragma unroll 1
      for (int q4 = 0; q4 < 4; ++q4) {
        float f[32], kf[32];
        ld32(tl + q4 * 32, f);
#pragma unroll
        for (int m = 0; m < 4; ++m) get_row_f(sK, i, q4 * 4 + m, kf + 8 * m);
        uint32_t r[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          part = fmaf(f[e], kf[e], part);
          r[e] = __float_as_uint(Bi * egi * f[e]);
        }
        tmem_st_32x32b_x32(tl + q4 * 32, r);  // dk accumulates on top of beta e^G T^T dW
      }
      tmem_wait_st();
      dB_own += egi * part;
      dG_own += Bi * egi * part;
#pragma unroll 1
      for (int h2 = 0; h2 < 2; ++h2) {
        float f[32], x[32];
        ld32(tl + 128 + h2 * 32, f);
        const float4* dd = reinterpret_cast<const float4*>(a.dDV + (ch * C + i) * C + h2 * 32);
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const float4 v4 = dd[m];
          const float dv4[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int j = h2 * 32 + 4 * m + u;
            x[4 * m + u] = Bs[j] * (__expf(Gs[j]) * f[4 * m + u] + dv4[u]);
          }
        }
#pragma unroll
        for (int m = 0; m < 4; ++m) put8(sX2, i, h2 * 4 + m, pack8(x + 8 * m));
      }
    }
  }
  fence_proxy_async();
  tc_fence_before();
  ok = __syncthreads_and(ok);

  // ---- D3 = T^T X2 -> Z
  if (ok && tid == 0) {
    tc_fence_after();
#pragma unroll
    for (int k = 0; k < 4; ++k)
      umma_bf16_ss(tmem + 192, mnmaj(aT, k), mnmaj(aX2, k), make_idesc_bf16(128, 64, 1, 1), k > 0);
    umma_commit(&bars[2]);
  }
  if (owner) {
    ok = __all_sync(0xffffffffu, ok && mbar_wait_bounded(&bars[2], 0, nullptr, args.status, kTimeoutEpilogue));
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int h2 = 0; h2 < 2; ++h2) {
        float f[32];
        ld32(tl + 192 + h2 * 32, f);
#pragma unroll
        for (int m = 0; m < 4; ++m) put8(sZ, i, h2 * 4 + m, pack8(f + 8 * m));
      }
    }
  }
  fence_proxy_async();
  tc_fence_before();
  ok = __syncthreads_and(ok);

  // ---- D4 = Z T^T -> dL (strictly lower), X1 = dL beta_i E, X3 = s dAqk o E
  if (ok && tid == 0) {
    tc_fence_after();
#pragma unroll
    for (int k = 0; k < 4; ++k)
      umma_bf16_ss(tmem + 128, kmaj(aZ, k), kmaj(aT, k), make_idesc_bf16(128, 64, 0, 0), k > 0);
    umma_commit(&bars[3]);
  }
  if (owner) {
    ok = __all_sync(0xffffffffu, ok && mbar_wait_bounded(&bars[3], 0, nullptr, args.status, kTimeoutEpilogue));
    if (ok) {
      tc_fence_after();
      float rb = 0.f, rg = 0.f;
#pragma unroll 1
      for (int h2 = 0; h2 < 2; ++h2) {
        // this row's k.k, s q.k (from the prep) and dAqk: independent 16-byte loads, all in flight
        float f[32], x3[32], kkr[32], qkr[32], dar[32];
        const float4* pk = reinterpret_cast<const float4*>(aux + i * C + h2 * 32);
        const float4* pq4 = reinterpret_cast<const float4*>(aux + C * C + i * C + h2 * 32);
        const float4* pa = reinterpret_cast<const float4*>(a.dAqk + (ch * C + i) * C + h2 * 32);
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const float4 x = pk[m], y = pq4[m], z = pa[m];
          kkr[4 * m] = x.x; kkr[4 * m + 1] = x.y; kkr[4 * m + 2] = x.z; kkr[4 * m + 3] = x.w;
          qkr[4 * m] = y.x; qkr[4 * m + 1] = y.y; qkr[4 * m + 2] = y.z; qkr[4 * m + 3] = y.w;
          dar[4 * m] = z.x; dar[4 * m + 1] = z.y; dar[4 * m + 2] = z.z; dar[4 * m + 3] = z.w;
        }
        ld32(tl + 128 + h2 * 32, f);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int j = h2 * 32 + e;
          const float dl = j < i ? -f[e] : 0.f;
          const float ex = j <= i ? __expf(Gi - Gs[j]) : 0.f;
          const float kk = kkr[e];
          const float x1 = dl * Bi * ex;
          rb = fmaf(dl * ex, kk, rb);
          const float m = x1 * kk;
          const float daq = j <= i ? dar[e] : 0.f;
          const float xq = daq * ex;
          const float pq = xq * qkr[e];
          rg += m + pq;
          Mc[sk(i, j)] = -(m + pq);
          X1s[sk(i, j)] = x1;
          x3[e] = a.scale * xq;
        }
#pragma unroll
        for (int m = 0; m < 4; ++m) put8(sX3, i, h2 * 4 + m, pack8(x3 + 8 * m));
      }
      dB_own += rb;
      dG_own += rg;
    }
    named_bar_sync(1, 64);
    if (ok) {
      // symmetric part of dKK: X1 + X1^T
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        float x[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const int j = cc * 8 + m;
          x[m] = X1s[sk(i, j)] + X1s[sk(j, i)];
        }
        put8(sXS, i, cc, pack8(x));
      }
    }
  }
  fence_proxy_async();
  tc_fence_before();
  ok = __syncthreads_and(ok);

  // ---- D5 += (X1 + X1^T) k + X3^T q, D6 = X3 k
  if (ok && tid == 0) {
    tc_fence_after();
#pragma unroll
    for (int k = 0; k < 4; ++k) umma_bf16_ss(tmem, kmaj(aXS, k), mnmaj(aK, k), make_idesc_bf16(128, 128, 0, 1), 1);
#pragma unroll
    for (int k = 0; k < 4; ++k) umma_bf16_ss(tmem, mnmaj(aX3, k), mnmaj(aQ, k), make_idesc_bf16(128, 128, 1, 1), 1);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      umma_bf16_ss(tmem + 128, kmaj(aX3, k), mnmaj(aK, k), make_idesc_bf16(128, 128, 0, 1), k > 0);
    umma_commit(&bars[4]);
  }
  if (!owner && ok) {
    // column sums of the dG contributions (rows of Mc are complete after the last barrier)
    const int j = tid - 64;
    float s = 0.f;
#pragma unroll 8
    for (int r = 0; r < C; ++r) s += Mc[sk(r, j)];
    dGc[j] = s;
  }
  if (owner) {
    ok = __all_sync(0xffffffffu, ok && mbar_wait_bounded(&bars[4], 0, nullptr, args.status, kTimeoutEpilogue));
    if (ok) {
      tc_fence_after();
      const float ed = __expf(GL - Gi);
      float qpart = 0.f, kpart = 0.f;
      const long off = ((long)(t0 + i) * H + h) * DK;
#pragma unroll 1
      for (int q4 = 0; q4 < 4; ++q4) {
        float d5[32], d6[32], kf[32], qf[32];
        ld32(tl + q4 * 32, d5);
        ld32(tl + 128 + q4 * 32, d6);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          get_row_f(sK, i, q4 * 4 + m, kf + 8 * m);
          get_row_f(sQ, i, q4 * 4 + m, qf + 8 * m);
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const long col = (ch * DK + q4 * 32 + e) * C + i;
          const float wk = a.dKdT[col], wq = a.dQgT[col];
          kpart = fmaf(wk, kf[e], kpart);
          qpart = fmaf(wq, qf[e], qpart);
          d5[e] = fmaf(ed, wk, d5[e]);
          d6[e] = fmaf(a.scale * egi, wq, d6[e]);
        }
        if (i < n) {
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            reinterpret_cast<uint4*>(a.dk + off + q4 * 32)[m] = pack8(d5 + 8 * m);
            reinterpret_cast<uint4*>(a.dq + off + q4 * 32)[m] = pack8(d6 + 8 * m);
          }
        }
      }
      dG_own += egi * a.scale * qpart;
      kpart *= ed;
      dG_own -= kpart;
      atomicAdd(&misc[0], kpart);
    }
  }
  // ---- D7 = T^T dDelta, once D5 / D6 are read and blocks 5-8 are free: dDelta^T arrives there
  fence_proxy_async();
  tc_fence_before();
  ok = __syncthreads_and(ok);
  bool dd_issued = false;
  if (ok && tid == 0) {
    mbar_arrive_expect_tx(&bars[6], nvb * BLK);
    for (int b = 0; b < nvb; ++b) tma_load_2d(sDD + b * BLK, &mDD, &bars[6], 0, (int)(ch * DV) + b * 64);
    dd_issued = true;
    if (mbar_wait_bounded(&bars[6], 0, nullptr, args.status, kTimeoutProducer)) {
      dd_issued = false;
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < 4; ++k)
        umma_bf16_ss(tmem, mnmaj(aT, k), kmaj(aDD, k), make_idesc_bf16(128, DV, 1, 0), k > 0);
      umma_commit(&bars[5]);
    }
  }
  if (owner) {
    ok = __all_sync(0xffffffffu, ok && mbar_wait_bounded(&bars[5], 0, nullptr, args.status, kTimeoutEpilogue));
    if (ok) {
      tc_fence_after();
      const long off = ((long)(t0 + i) * H + h) * DV;
#pragma unroll 1
      for (int q = 0; q < DV / 32; ++q) {
        float d7[32];
        ld32(tl + q * 32, d7);
        if (i < n) {
          float vv[32], o[32];
#pragma unroll
          for (int m = 0; m < 4; ++m) unpack8(reinterpret_cast<const uint4*>(a.v + off + q * 32)[m], vv + 8 * m);
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            dB_own = fmaf(d7[e], vv[e], dB_own);
            o[e] = Bi * d7[e];
          }
#pragma unroll
          for (int m = 0; m < 4; ++m) reinterpret_cast<uint4*>(a.dv + off + q * 32)[m] = pack8(o + 8 * m);
        }
      }
    }
  }
  ok = __syncthreads_and(ok);
  // ---- dg = reverse cumulative sum of dG over the chunk; dbeta
  float* dGt = X1s;
  float* dBt = X1s + C;
  if (owner) {
    float t = dG_own + dGc[i];
    if (i == C - 1) t += misc[0] + __expf(GL) * a.dgam[ch];
    dGt[i] = t;
    dBt[i] = dB_own;
  }
  __syncthreads();
  if (ok && tid < 32) {
    float x0 = dGt[tid], x1 = dGt[tid + 32];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y0 = __shfl_down_sync(0xffffffffu, x0, o);
      const float y1 = __shfl_down_sync(0xffffffffu, x1, o);
      if (tid + o < 32) {
        x0 += y0;
        x1 += y1;
      }
    }
    x0 += __shfl_sync(0xffffffffu, x1, 0);
    if (tid < n) {
      a.dg[(long)(t0 + tid) * H + h] = x0;
      a.dbeta[(long)(t0 + tid) * H + h] = dBt[tid];
    }
    if (tid + 32 < n) {
      a.dg[(long)(t0 + tid + 32) * H + h] = x1;
      a.dbeta[(long)(t0 + tid + 32) * H + h] = dBt[tid + 32];
    }
  }
  if (tid == 0 && !ok) {
    // no TMA copy may outlive the CTA
    mbar_wait_bounded(&bars[0], 0, nullptr, nullptr, 0);
    if (dd_issued) mbar_wait_bounded(&bars[6], 0, nullptr, nullptr, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ============================================================================ host
CUtensorMap map2d(const at::Tensor& t, int64_t rows, int64_t cols, int64_t row_stride) {
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, "gdn: bf16 tensor expected");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0 && row_stride % 8 == 0,
              "gdn: tensors must be 16-byte aligned with 16-byte row strides");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, t.data_ptr(), dims, strides, box, estr,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) tma_encode_failed("gdn map", (int)r, t.data_ptr(), 2, dims, strides, box);
  return m;
}

void check_bf16(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), "gdn: ", name,
              " must be a contiguous bf16 CUDA tensor");
}

void check_f32(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous(), "gdn: ", name,
              " must be a contiguous fp32 CUDA tensor");
}

}  // namespace gdnc

// q, k [T, H, 128], v [T, H, DV] bf16; g, beta [T, H] fp32; tok0/len [Nc] int32.
std::vector<at::Tensor> gdn_chunk_prep(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                       const at::Tensor& g, const at::Tensor& beta, const at::Tensor& tok0,
                                       const at::Tensor& len, double scale, bool with_aux, at::Tensor& status) {
  using namespace gdnc;
  check_bf16(q, "q");
  check_bf16(k, "k");
  check_bf16(v, "v");
  check_f32(g, "g");
  check_f32(beta, "beta");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == DK && k.sizes() == q.sizes(), "gdn: q/k must be [T, H, 128]");
  const int H = q.size(1), DV = v.size(2);
  TORCH_CHECK(DV % 128 == 0 && DV <= 256 && v.size(0) == q.size(0) && v.size(1) == H,
              "gdn: v must be [T, H, DV] with DV in {128, 256}");
  const int Nc = tok0.numel();
  const c10::cuda::CUDAGuard guard(q.device());
  auto bf = q.options();
  auto f32 = q.options().dtype(at::kFloat);
  at::Tensor Wn = at::empty({Nc, H, C, DK}, bf), U = at::empty({Nc, H, C, DV}, bf);
  at::Tensor Kd = at::empty({Nc, H, C, DK}, bf), Qg = at::empty({Nc, H, C, DK}, bf);
  at::Tensor Aqk = at::empty({Nc, H, C, C}, bf);
  at::Tensor gam = at::empty({Nc, H}, f32), Gc = at::empty({Nc, H, C}, f32);
  at::Tensor aux = with_aux ? at::empty({Nc, H, 3, C, C}, f32) : at::empty({0}, f32);
  if (Nc == 0) return {Wn, U, Kd, Qg, Aqk, gam, Gc, aux};
  const int64_t T = q.size(0);
  TORCH_CHECK(T >= C, "gdn: at least 64 tokens");
  CUtensorMap mQ = map2d(q, T, (int64_t)H * DK, (int64_t)H * DK), mK = map2d(k, T, (int64_t)H * DK, (int64_t)H * DK);
  CUtensorMap mV = map2d(v, T, (int64_t)H * DV, (int64_t)H * DV);
  PrepTcParams a{g.data_ptr<float>(), beta.data_ptr<float>(), tok0.data_ptr<int>(), len.data_ptr<int>(),
                 reinterpret_cast<__nv_bfloat16*>(Wn.data_ptr()), reinterpret_cast<__nv_bfloat16*>(U.data_ptr()),
                 reinterpret_cast<__nv_bfloat16*>(Kd.data_ptr()), reinterpret_cast<__nv_bfloat16*>(Qg.data_ptr()),
                 reinterpret_cast<__nv_bfloat16*>(Aqk.data_ptr()), gam.data_ptr<float>(), Gc.data_ptr<float>(),
                 with_aux ? aux.data_ptr<float>() : nullptr, (float)scale, H, DV, status.data_ptr<int>()};
  const int smem = prep_tc_smem(DV);
  static int attr = 0;
  if (attr < smem) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gdn_prep_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr = smem;
  }
  gdn_prep_tc_kernel<<<Nc * H, TP_THREADS, smem, at::cuda::getCurrentCUDAStream()>>>(mQ, mK, mV, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {Wn, U, Kd, Qg, Aqk, gam, Gc, aux};
}

namespace gdnc {
template <bool BWD>
void launch_state(const at::Tensor& Wn, const at::Tensor& Qg, const at::Tensor& Kd, const at::Tensor& Aqk,
                  const at::Tensor& X, const StateParams& p, int nseq, int Nc) {
  const int H = p.H, DV = p.DV;
  const int64_t rows = (int64_t)Nc * H * C;
  CUtensorMap mWn = map2d(Wn, rows, DK, DK), mQg = map2d(Qg, rows, DK, DK), mKd = map2d(Kd, rows, DK, DK);
  CUtensorMap mAqk = map2d(Aqk, rows, C, C);
  CUtensorMap mX = BWD ? map2d(X, X.size(0), (int64_t)H * DV, (int64_t)H * DV) : map2d(X, rows, DV, DV);
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gdn_state_tc_kernel<BWD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        ST_SMEM));
    attr = true;
  }
  dim3 grid(nseq, H, DV / VS);
  gdn_state_tc_kernel<BWD><<<grid, ST_THREADS, ST_SMEM, at::cuda::getCurrentCUDAStream()>>>(mWn, mQg, mKd, mAqk,
                                                                                             mX, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

const float* opt_f32(const c10::optional<at::Tensor>& t) {
  if (!t.has_value() || !t->defined()) return nullptr;
  check_f32(*t, "state");
  return t->data_ptr<float>();
}
}  // namespace gdnc

// Forward state pass with the output fused. Returns nothing; writes `out` (o),
// `S_final`, and optionally the per-chunk states S_c^T and Delta_c^T.
void gdn_chunk_fwd(const at::Tensor& Wn, const at::Tensor& U, const at::Tensor& Kd, const at::Tensor& Qg,
                   const at::Tensor& Aqk, const at::Tensor& gam, const at::Tensor& tok0, const at::Tensor& len,
                   const at::Tensor& seq_chunks, const c10::optional<at::Tensor>& S0,
                   const c10::optional<at::Tensor>& out, const c10::optional<at::Tensor>& S_final,
                   const c10::optional<at::Tensor>& states, const c10::optional<at::Tensor>& rows,
                   at::Tensor& status) {
  using namespace gdnc;
  const int Nc = Wn.size(0), H = Wn.size(1), DV = U.size(3);
  const int nseq = seq_chunks.numel() - 1;
  const c10::cuda::CUDAGuard guard(Wn.device());
  StateParams p{};
  p.seq_chunks = seq_chunks.data_ptr<int>();
  p.tok0 = tok0.data_ptr<int>();
  p.len = len.data_ptr<int>();
  p.gam = gam.data_ptr<float>();
  p.S_in = opt_f32(S0);
  p.S_out = S_final.has_value() && S_final->defined() ? S_final->data_ptr<float>() : nullptr;
  p.states = states.has_value() && states->defined() ? reinterpret_cast<__nv_bfloat16*>(states->data_ptr()) : nullptr;
  p.rows = rows.has_value() && rows->defined() ? reinterpret_cast<__nv_bfloat16*>(rows->data_ptr()) : nullptr;
  p.out = out.has_value() && out->defined() ? reinterpret_cast<__nv_bfloat16*>(out->data_ptr()) : nullptr;
  if (p.out != nullptr) check_bf16(*out, "out");
  p.T = p.out != nullptr ? (int)out->size(0) : 0;
  p.H = H;
  p.DV = DV;
  p.status = status.data_ptr<int>();
  if (nseq == 0 || Nc == 0) return;
  launch_state<false>(Wn, Qg, Kd, Aqk, U, p, nseq, Nc);
}

// Reverse state pass: writes G_{c+1}^T per chunk (`states`), dDelta_c^T (`rows`)
// and the gradient of the initial state (`dS0`, optional).
void gdn_chunk_bwd_state(const at::Tensor& Wn, const at::Tensor& Kd, const at::Tensor& Qg, const at::Tensor& Aqk,
                         const at::Tensor& gam, const at::Tensor& dout, const at::Tensor& tok0, const at::Tensor& len,
                         const at::Tensor& seq_chunks, const c10::optional<at::Tensor>& dS_final,
                         const c10::optional<at::Tensor>& dS0, at::Tensor& states, at::Tensor& rows,
                         at::Tensor& status) {
  using namespace gdnc;
  check_bf16(dout, "dout");
  const int Nc = Wn.size(0), H = Wn.size(1), DV = dout.size(2);
  const int nseq = seq_chunks.numel() - 1;
  const c10::cuda::CUDAGuard guard(Wn.device());
  StateParams p{};
  p.seq_chunks = seq_chunks.data_ptr<int>();
  p.tok0 = tok0.data_ptr<int>();
  p.len = len.data_ptr<int>();
  p.gam = gam.data_ptr<float>();
  p.S_in = opt_f32(dS_final);
  p.S_out = dS0.has_value() && dS0->defined() ? dS0->data_ptr<float>() : nullptr;
  p.states = reinterpret_cast<__nv_bfloat16*>(states.data_ptr());
  p.rows = reinterpret_cast<__nv_bfloat16*>(rows.data_ptr());
  p.out = nullptr;
  p.H = H;
  p.DV = DV;
  p.status = status.data_ptr<int>();
  if (nseq == 0 || Nc == 0) return;
  launch_state<true>(Wn, Qg, Kd, Aqk, dout.view({dout.size(0), (int64_t)H * DV}), p, nseq, Nc);
}

// Which chunk-local backward runs: the tensor-core kernel (default) or the CUDA-core kernel
// (PRISM_GDN_LOCAL_TC=0, or gdn_local_tc_enabled(0)); `set` < 0 only queries.
bool gdn_local_tc_enabled(int64_t set) {
  static int state = [] {
    const char* e = getenv("PRISM_GDN_LOCAL_TC");
    return (e == nullptr || strcmp(e, "0") != 0) ? 1 : 0;
  }();
  if (set >= 0) state = set != 0;
  return state != 0;
}

// Chunk-local backward: dv-contractions on tcgen05, then the WY/decay backward.
// `second` (optional): {states, dstates, rows, drows, dout} of a second state pass with zero values
// over the first states.size(0) chunks (the same prep, dv = dk): its contractions are added to the
// first pass's before the local backward (it adds nothing through the values, which are zero).
std::vector<at::Tensor> gdn_chunk_bwd_local(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                            const at::Tensor& g, const at::Tensor& beta, const at::Tensor& tok0,
                                            const at::Tensor& len, const at::Tensor& Gc, const at::Tensor& aux,
                                            const at::Tensor& states,
                                            const at::Tensor& dstates, const at::Tensor& rows,
                                            const at::Tensor& drows, const at::Tensor& dout, double scale,
                                            at::Tensor& status, const std::vector<at::Tensor>& second) {
  using namespace gdnc;
  const int Nc = tok0.numel(), H = q.size(1), DV = v.size(2);
  const c10::cuda::CUDAGuard guard(q.device());
  auto f32 = q.options().dtype(at::kFloat);
  at::Tensor dWnT = at::empty({Nc, H, DK, C}, f32), dQgT = at::empty({Nc, H, DK, C}, f32);
  at::Tensor dKdT = at::empty({Nc, H, DK, C}, f32), dAqk = at::empty({Nc, H, C, C}, f32);
  at::Tensor dDV = at::empty({Nc, H, C, C}, f32), dgam = at::empty({Nc, H}, f32);
  at::Tensor dq = at::empty_like(q), dk = at::empty_like(k), dv = at::empty_like(v);
  at::Tensor dg = at::empty_like(g), dbeta = at::empty_like(beta);
  if (Nc == 0) return {dq, dk, dv, dg, dbeta};
  const int64_t srows = (int64_t)Nc * H * DV;
  CUtensorMap mS = map2d(states, srows, DK, DK), mG = map2d(dstates, srows, DK, DK);
  CUtensorMap mDL = map2d(rows, srows, C, C), mDD = map2d(drows, srows, C, C);
  CUtensorMap mDO = map2d(dout, dout.size(0), (int64_t)H * DV, (int64_t)H * DV);
  CUtensorMap mV = map2d(v, v.size(0), (int64_t)H * DV, (int64_t)H * DV);
  DvParams dp{tok0.data_ptr<int>(), dWnT.data_ptr<float>(), dQgT.data_ptr<float>(), dKdT.data_ptr<float>(),
              dAqk.data_ptr<float>(), dDV.data_ptr<float>(), dgam.data_ptr<float>(), H, DV, status.data_ptr<int>(), 0};
  const int dv_smem = DV * 896 + 128 + 1024;
  static int attr_dv = 0;
  if (attr_dv < dv_smem) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gdn_bwd_dv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dv_smem));
    attr_dv = dv_smem;
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  gdn_bwd_dv_kernel<<<Nc * H, DV_THREADS, dv_smem, stream>>>(mS, mG, mDO, mDD, mDL, mV, dp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (!second.empty()) {
    TORCH_CHECK(second.size() == 5, "gdn_chunk_bwd_local: second pass = {states, dstates, rows, drows, dout}");
    const at::Tensor &s2 = second[0], &g2 = second[1], &r2 = second[2], &dr2 = second[3], &do2 = second[4];
    check_bf16(do2, "second dout");
    const int Nc2 = s2.size(0), DV2 = s2.size(2);
    TORCH_CHECK(Nc2 <= Nc && s2.size(1) == H && DV2 == DK && do2.size(2) == DV2,
                "gdn_chunk_bwd_local: the second pass covers the first chunks with dv = dk");
    const int64_t srows2 = (int64_t)Nc2 * H * DV2;
    CUtensorMap mS2 = map2d(s2, srows2, DK, DK), mG2 = map2d(g2, srows2, DK, DK);
    CUtensorMap mDL2 = map2d(r2, srows2, C, C), mDD2 = map2d(dr2, srows2, C, C);
    CUtensorMap mDO2 = map2d(do2, do2.size(0), (int64_t)H * DV2, (int64_t)H * DV2);
    DvParams dp2 = dp;
    dp2.DV = DV2;
    dp2.dDV = nullptr;  // dDelta V^T with zero values
    dp2.accumulate = 1;
    const int dv_smem2 = DV2 * 896 + 128 + 1024;
    if (attr_dv < dv_smem2) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(gdn_bwd_dv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dv_smem2));
      attr_dv = dv_smem2;
    }
    gdn_bwd_dv_kernel<<<Nc2 * H, DV_THREADS, dv_smem2, stream>>>(mS2, mG2, mDO2, mDD2, mDL2, mDO2, dp2);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  LocalArgs la{reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()),
               reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()), g.data_ptr<float>(), beta.data_ptr<float>(),
               tok0.data_ptr<int>(), len.data_ptr<int>(), Gc.data_ptr<float>(), aux.data_ptr<float>(),
               dWnT.data_ptr<float>(),
               dQgT.data_ptr<float>(), dKdT.data_ptr<float>(), dAqk.data_ptr<float>(), dDV.data_ptr<float>(),
               dgam.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(drows.data_ptr()),
               reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dk.data_ptr()),
               reinterpret_cast<__nv_bfloat16*>(dv.data_ptr()), dg.data_ptr<float>(), dbeta.data_ptr<float>(),
               (float)scale, H, DV};
  if (gdn_local_tc_enabled(-1)) {
    const int64_t T = q.size(0);
    CUtensorMap mQ = map2d(q, T, (int64_t)H * DK, (int64_t)H * DK), mK = map2d(k, T, (int64_t)H * DK, (int64_t)H * DK);
    static bool attr_tc = false;
    if (!attr_tc) {
      C10_CUDA_CHECK(
          cudaFuncSetAttribute(gdn_bwd_local_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, lt::SMEM));
      attr_tc = true;
    }
    gdn_bwd_local_tc_kernel<<<Nc * H, lt::THREADS, lt::SMEM, stream>>>(mQ, mK, mDD, LocalTcArgs{la, status.data_ptr<int>()});
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return {dq, dk, dv, dg, dbeta};
  }
  static bool attr_lb = false;
  if (!attr_lb) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gdn_bwd_local_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, LB_SMEM));
    attr_lb = true;
  }
  gdn_bwd_local_kernel<<<Nc * H, LB_THREADS, LB_SMEM, stream>>>(la);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dq, dk, dv, dg, dbeta};
}

}  // namespace prism
