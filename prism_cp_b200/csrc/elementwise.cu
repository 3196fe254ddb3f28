// Memory-bound kernels of the hybrid decoder: RoPE, causal depthwise conv1d +
// SiLU (with a cross-rank halo for contiguous context parallelism), SwiGLU,
// fused softmax cross-entropy (loss and logit gradient in one pass pair),
// AdamW over flat fp32 shards and the squared gradient norm.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace prism {
namespace {

__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void st8(__nv_bfloat16* p, const float (&f)[8]) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                            pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
}

// ------------------------------------------------------------------ RoPE
// Rotate-half RoPE in place on x viewed as [T, heads, d] with row stride `stride`.
// sign = +1 forward, -1 backward (inverse rotation).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ x, long stride, const int* __restrict__ pos, int T, int heads,
                            int d, float log2_base, float sign) {
  const int half = d / 2;
  const int groups = half / 8;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long total = (long)T * heads * groups;
  if (idx >= total) return;
  const int g = idx % groups;
  const long th = idx / groups;
  const int h = th % heads;
  const long t = th / heads;
  __nv_bfloat16* row = x + t * stride + (long)h * d;
  float a[8], b[8];
  ld8(row + g * 8, a);
  ld8(row + half + g * 8, b);
  const float p = (float)pos[t];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int i = g * 8 + e;
    const float inv_freq = exp2f(-(2.0f * i / d) * log2_base);
    float s, c;
    sincosf(p * inv_freq, &s, &c);
    s *= sign;
    const float x1 = a[e], x2 = b[e];
    a[e] = x1 * c - x2 * s;
    b[e] = x2 * c + x1 * s;
  }
  st8(row + g * 8, a);
  st8(row + half + g * 8, b);
}

// ------------------------------------------------------------------ conv1d
constexpr int kConvTok = 64;  // tokens per thread block
constexpr int kConvK = 4;

__device__ __forceinline__ int find_segment(const int* cu, int nseg, int t) {
  int lo = 0, hi = nseg - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__global__ void conv_fwd_kernel(const __nv_bfloat16* __restrict__ x, long xs, const __nv_bfloat16* __restrict__ w,
                                const __nv_bfloat16* __restrict__ halo, const int* __restrict__ cu, int nseg, int T,
                                int C, __nv_bfloat16* __restrict__ y, float* __restrict__ pre_out) {
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int t0 = blockIdx.x * kConvTok;
  const int t1 = min(T, t0 + kConvTok);
  float wk[kConvK];
#pragma unroll
  for (int j = 0; j < kConvK; ++j) wk[j] = __bfloat162float(w[c * kConvK + j]);
  int seg = find_segment(cu, nseg, t0);
  for (int t = t0; t < t1; ++t) {
    while (seg + 1 < nseg && cu[seg + 1] <= t) ++seg;
    const int start = cu[seg];
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < kConvK; ++j) {
      const int u = t - (kConvK - 1) + j;
      float v = 0.f;
      if (u >= start) v = __bfloat162float(x[(long)u * xs + c]);
      else if (seg == 0 && halo != nullptr) v = __bfloat162float(halo[(long)(u - start + kConvK - 1) * C + c]);
      acc += wk[j] * v;
    }
    y[(long)t * C + c] = __float2bfloat16(silu(acc));
  }
}

// dx[t] = sum_j w[j] * dpre[t + 3 - j] (same segment); dw[j] += dpre[t] * x[t - 3 + j];
// dhalo[t + j] += w[j] * dpre[t] where t - 3 + j falls before segment 0.
__global__ void conv_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x, long xs,
                                const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ halo,
                                const int* __restrict__ cu, int nseg, int T, int C, __nv_bfloat16* __restrict__ dx,
                                long dxs, float* __restrict__ dw, float* __restrict__ dhalo) {
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int t0 = blockIdx.x * kConvTok;
  const int t1 = min(T, t0 + kConvTok);
  float wk[kConvK];
#pragma unroll
  for (int j = 0; j < kConvK; ++j) wk[j] = __bfloat162float(w[c * kConvK + j]);
  auto xval = [&](int seg, int start, int u) -> float {
    if (u >= start) return __bfloat162float(x[(long)u * xs + c]);
    if (seg == 0 && halo != nullptr) return __bfloat162float(halo[(long)(u - start + kConvK - 1) * C + c]);
    return 0.f;
  };
  auto dpre_at = [&](int s) -> float {
    // s must be a valid token index
    const int seg = find_segment(cu, nseg, s);
    const int start = cu[seg];
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < kConvK; ++j) acc += wk[j] * xval(seg, start, s - (kConvK - 1) + j);
    const float sg = sigmoidf_(acc);
    return __bfloat162float(dy[(long)s * C + c]) * sg * (1.f + acc * (1.f - sg));
  };
  float dwacc[kConvK] = {0.f, 0.f, 0.f, 0.f};
  float dh[kConvK - 1] = {0.f, 0.f, 0.f};
  for (int t = t0; t < t1; ++t) {
    const int seg = find_segment(cu, nseg, t);
    const int start = cu[seg], end = cu[seg + 1];
    // own dpre for dw / dhalo
    const float dp = dpre_at(t);
#pragma unroll
    for (int j = 0; j < kConvK; ++j) {
      const int u = t - (kConvK - 1) + j;
      dwacc[j] += dp * xval(seg, start, u);
      if (u < start && seg == 0 && halo != nullptr) dh[u - start + kConvK - 1] += wk[j] * dp;
    }
    // gather dx[t]
    float acc = wk[kConvK - 1] * dp;
#pragma unroll
    for (int j = 0; j < kConvK - 1; ++j) {
      const int s = t + (kConvK - 1) - j;
      if (s < end) acc += wk[j] * dpre_at(s);
    }
    dx[(long)t * dxs + c] = __float2bfloat16(acc);
  }
#pragma unroll
  for (int j = 0; j < kConvK; ++j) atomicAdd(&dw[c * kConvK + j], dwacc[j]);
  if (dhalo != nullptr && halo != nullptr && t0 < cu[min(1, nseg)]) {
#pragma unroll
    for (int j = 0; j < kConvK - 1; ++j) atomicAdd(&dhalo[(long)j * C + c], dh[j]);
  }
}

// Vectorised forms: one thread owns 8 consecutive channels (16-byte loads) and
// walks kConvTokV tokens with the last three inputs (forward) or pre-activation
// gradients (backward) held in registers, so every x and dy element is read once
// per pass instead of once per tap. Used when C % 8 == 0 and rows are 16-byte
// aligned; dx[t] = sum_j w[j] dpre[t + 3 - j] is finalised when dpre[t + 3]
// is known, or at a segment end with the missing terms zero.
constexpr int kConvTokV = 256;

__device__ __forceinline__ void ld8f(const __nv_bfloat16* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void st8f(__nv_bfloat16* p, const float* f) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                            pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
}

// x value of token u for a sequence starting at `start` (halo rows before sequence 0)
__device__ __forceinline__ void conv_x8(const __nv_bfloat16* x, long xs, const __nv_bfloat16* halo, int C, int c8,
                                        int seg, int start, int u, float* f) {
  if (u >= start) {
    ld8f(x + (long)u * xs + c8, f);
  } else if (seg == 0 && halo != nullptr && u - start + kConvK - 1 >= 0) {
    ld8f(halo + (long)(u - start + kConvK - 1) * C + c8, f);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = 0.f;
  }
}

__global__ void conv_fwd_vec_kernel(const __nv_bfloat16* __restrict__ x, long xs, const __nv_bfloat16* __restrict__ w,
                                    const __nv_bfloat16* __restrict__ halo, const int* __restrict__ cu, int nseg,
                                    int T, int C, __nv_bfloat16* __restrict__ y) {
  const int c8 = 8 * (blockIdx.y * blockDim.x + threadIdx.x);
  if (c8 >= C) return;
  const int t0 = blockIdx.x * kConvTokV;
  const int t1 = min(T, t0 + kConvTokV);
  float wk[8][kConvK];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < kConvK; ++j) wk[i][j] = __bfloat162float(w[(c8 + i) * kConvK + j]);
  int seg = find_segment(cu, nseg, t0);
  int start = cu[seg], end = cu[seg + 1];
  float xm3[8], xm2[8], xm1[8];
  conv_x8(x, xs, halo, C, c8, seg, start, t0 - 3, xm3);
  conv_x8(x, xs, halo, C, c8, seg, start, t0 - 2, xm2);
  conv_x8(x, xs, halo, C, c8, seg, start, t0 - 1, xm1);
  for (int t = t0; t < t1; ++t) {
    if (t == end) {
      while (seg + 1 < nseg && cu[seg + 1] <= t) ++seg;
      start = cu[seg];
      end = cu[seg + 1];
#pragma unroll
      for (int i = 0; i < 8; ++i) xm3[i] = xm2[i] = xm1[i] = 0.f;
    }
    float xt[8], out[8];
    ld8f(x + (long)t * xs + c8, xt);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float acc = wk[i][0] * xm3[i] + wk[i][1] * xm2[i] + wk[i][2] * xm1[i] + wk[i][3] * xt[i];
      out[i] = silu(acc);
      xm3[i] = xm2[i];
      xm2[i] = xm1[i];
      xm1[i] = xt[i];
    }
    st8f(y + (long)t * C + c8, out);
  }
}

// Token-parallel forward: thread (channel group, token) computes one 8-channel output row
// from its four taps. A warp covers 32 consecutive channel groups of one token (512
// contiguous bytes per row); a block covers 32 channel groups x 128 tokens, each thread
// 16 tokens 8 apart, four at a time. No sequential chain, so every load is independent and in flight
// at once; the taps' rows are shared through L1/L2, DRAM traffic stays one read of x
// and one write of y.
constexpr int kConvTokP = 128;
constexpr bool kConvTokenParallel = true;  // false: the sequential 256-token form above

__global__ void __launch_bounds__(256) conv_fwd_tok_kernel(const __nv_bfloat16* __restrict__ x, long xs,
                                                           const __nv_bfloat16* __restrict__ w,
                                                           const __nv_bfloat16* __restrict__ halo,
                                                           const int* __restrict__ cu, int nseg, int T, int C,
                                                           __nv_bfloat16* __restrict__ y) {
  const int tc = threadIdx.x & 31, tt = threadIdx.x >> 5;
  const int c8 = 8 * (blockIdx.y * 32 + tc);
  if (c8 >= C) return;
  float wk[8][kConvK];
  {
    // 8 channels x 4 taps = 32 consecutive bf16 (64 bytes)
    const uint4* wp = reinterpret_cast<const uint4*>(w + (long)c8 * kConvK);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float f[8];
      ld8f(reinterpret_cast<const __nv_bfloat16*>(wp + q), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) wk[2 * q + e / 4][e % 4] = f[e];
    }
  }
#pragma unroll 4
  for (int k = 0; k < kConvTokP / 8; ++k) {
    const int t = blockIdx.x * kConvTokP + tt + 8 * k;
    if (t >= T) continue;  // predicated, so the unrolled iterations' loads can all be in flight
    const int seg = find_segment(cu, nseg, t);
    const int start = cu[seg];
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < kConvK; ++j) {
      float f[8];
      conv_x8(x, xs, halo, C, c8, seg, start, t - (kConvK - 1) + j, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(wk[i][j], f[i], acc[i]);
    }
    float out[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = silu(acc[i]);
    st8f(y + (long)t * C + c8, out);
  }
}

__global__ void conv_bwd_vec_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                    long xs, const __nv_bfloat16* __restrict__ w,
                                    const __nv_bfloat16* __restrict__ halo, const int* __restrict__ cu, int nseg,
                                    int T, int C, __nv_bfloat16* __restrict__ dx, long dxs, float* __restrict__ dw,
                                    float* __restrict__ dhalo) {
  const int c8 = 8 * (blockIdx.y * blockDim.x + threadIdx.x);
  if (c8 >= C) return;
  const int t0 = blockIdx.x * kConvTokV;
  const int t1 = min(T, t0 + kConvTokV);
  const int s_end = min(T, t1 + kConvK - 1);
  float wk[8][kConvK];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < kConvK; ++j) wk[i][j] = __bfloat162float(w[(c8 + i) * kConvK + j]);
  int seg = find_segment(cu, nseg, t0);
  int start = cu[seg], end = cu[seg + 1];
  float xm3[8], xm2[8], xm1[8];
  conv_x8(x, xs, halo, C, c8, seg, start, t0 - 3, xm3);
  conv_x8(x, xs, halo, C, c8, seg, start, t0 - 2, xm2);
  conv_x8(x, xs, halo, C, c8, seg, start, t0 - 1, xm1);
  float dm3[8], dm2[8], dm1[8];
  float dwa[8][kConvK], dha[8][kConvK - 1];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    dm3[i] = dm2[i] = dm1[i] = 0.f;
#pragma unroll
    for (int j = 0; j < kConvK; ++j) dwa[i][j] = 0.f;
#pragma unroll
    for (int j = 0; j < kConvK - 1; ++j) dha[i][j] = 0.f;
  }
  // dx of tokens [lo, s) whose later taps fall past the segment end (or the data)
  auto flush = [&](int s, int lo) {
    for (int t = max(lo, s - 3); t < min(s, t1); ++t) {
      float out[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int k = s - t;  // 1..3 pending values: dpre[t..s-1]
        float acc;
        if (k == 3) acc = wk[i][3] * dm3[i] + wk[i][2] * dm2[i] + wk[i][1] * dm1[i];
        else if (k == 2) acc = wk[i][3] * dm2[i] + wk[i][2] * dm1[i];
        else acc = wk[i][3] * dm1[i];
        out[i] = acc;
      }
      st8f(dx + (long)t * dxs + c8, out);
    }
  };
  for (int s = t0; s < s_end; ++s) {
    if (s == end) {
      flush(s, max(t0, start));
      while (seg + 1 < nseg && cu[seg + 1] <= s) ++seg;
      start = cu[seg];
      end = cu[seg + 1];
#pragma unroll
      for (int i = 0; i < 8; ++i) xm3[i] = xm2[i] = xm1[i] = dm3[i] = dm2[i] = dm1[i] = 0.f;
    }
    float xt[8], g[8], dp[8];
    ld8f(x + (long)s * xs + c8, xt);
    ld8f(dy + (long)s * C + c8, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float acc = wk[i][0] * xm3[i] + wk[i][1] * xm2[i] + wk[i][2] * xm1[i] + wk[i][3] * xt[i];
      const float sg = sigmoidf_(acc);
      dp[i] = g[i] * sg * (1.f + acc * (1.f - sg));
    }
    if (s < t1) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dwa[i][0] += dp[i] * xm3[i];
        dwa[i][1] += dp[i] * xm2[i];
        dwa[i][2] += dp[i] * xm1[i];
        dwa[i][3] += dp[i] * xt[i];
      }
      if (seg == 0 && halo != nullptr && s - start < kConvK - 1) {
        // taps j with s - 3 + j < start read halo row s - start + j
#pragma unroll
        for (int j = 0; j < kConvK - 1; ++j) {
          const int hrow = s - start + j;
          if (hrow < kConvK - 1) {
#pragma unroll
            for (int i = 0; i < 8; ++i) dha[i][hrow] += wk[i][j] * dp[i];
          }
        }
      }
    }
    if (s - 3 >= max(t0, start)) {
      float out[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        out[i] = wk[i][3] * dm3[i] + wk[i][2] * dm2[i] + wk[i][1] * dm1[i] + wk[i][0] * dp[i];
      st8f(dx + (long)(s - 3) * dxs + c8, out);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xm3[i] = xm2[i];
      xm2[i] = xm1[i];
      xm1[i] = xt[i];
      dm3[i] = dm2[i];
      dm2[i] = dm1[i];
      dm1[i] = dp[i];
    }
  }
  if (s_end == T || s_end == end) flush(s_end, max(t0, start));
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < kConvK; ++j) atomicAdd(&dw[(c8 + i) * kConvK + j], dwa[i][j]);
  if (dhalo != nullptr && halo != nullptr && t0 < cu[min(1, nseg)]) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < kConvK - 1; ++j) atomicAdd(&dhalo[(long)j * C + c8 + i], dha[i][j]);
  }
}

// ------------------------------------------------------------------ SwiGLU
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ x, long xs, __nv_bfloat16* __restrict__ y,
                                  long ys, int T, int F) {
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int groups = F / 8;
  if (idx >= (long)T * groups) return;
  const long t = idx / groups;
  const int g = idx % groups;
  float a[8], b[8], o[8];
  ld8(x + t * xs + g * 8, a);
  ld8(x + t * xs + F + g * 8, b);
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = silu(a[e]) * b[e];
  st8(y + t * ys + g * 8, o);
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dy, long dys, const __nv_bfloat16* __restrict__ x,
                                  long xs, __nv_bfloat16* __restrict__ dx, long dxs, int T, int F) {
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int groups = F / 8;
  if (idx >= (long)T * groups) return;
  const long t = idx / groups;
  const int g = idx % groups;
  float a[8], b[8], d[8], da[8], db[8];
  ld8(x + t * xs + g * 8, a);
  ld8(x + t * xs + F + g * 8, b);
  ld8(dy + t * dys + g * 8, d);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float s = sigmoidf_(a[e]);
    db[e] = d[e] * a[e] * s;
    da[e] = d[e] * b[e] * s * (1.f + a[e] * (1.f - s));
  }
  st8(dx + t * dxs + g * 8, da);
  st8(dx + t * dxs + F + g * 8, db);
}

// ------------------------------------------------------------------ cross-entropy
// One block per row: loss[r] = lse - logit[label]; logits[r] <- weight[r] * (softmax - onehot).
constexpr int kCeThreads = 512;

__global__ void __launch_bounds__(kCeThreads) ce_fused_kernel(__nv_bfloat16* __restrict__ logits, long ls,
                                                              const int64_t* __restrict__ labels,
                                                              const float* __restrict__ weight, int V,
                                                              float* __restrict__ loss, float* __restrict__ lse_out) {
  __shared__ float red_m[kCeThreads / 32], red_s[kCeThreads / 32];
  const long r = blockIdx.x;
  __nv_bfloat16* row = logits + r * ls;
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x * 8; i < V; i += kCeThreads * 8) {
    float f[8];
    ld8(row + i, f);
    float lm = f[0];
#pragma unroll
    for (int e = 1; e < 8; ++e) lm = fmaxf(lm, f[e]);
    const float nm = fmaxf(m, lm);
    float acc = s * __expf(m - nm);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc += __expf(f[e] - nm);
    m = nm;
    s = acc;
  }
  // warp then block reduction of (max, sum)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
    m = nm;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red_m[warp] = m;
    red_s[warp] = s;
  }
  __syncthreads();
  if (warp == 0) {
    m = lane < kCeThreads / 32 ? red_m[lane] : -INFINITY;
    s = lane < kCeThreads / 32 ? red_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o);
      const float os = __shfl_xor_sync(0xffffffffu, s, o);
      const float nm = fmaxf(m, om);
      s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
      m = nm;
    }
    if (lane == 0) {
      red_m[0] = m;
      red_s[0] = s;
    }
  }
  __syncthreads();
  m = red_m[0];
  s = red_s[0];
  const float lse = m + logf(s);
  const int64_t label = labels[r];
  const float wgt = weight[r];
  if (threadIdx.x == 0) {
    const float target = (label >= 0 && label < V) ? __bfloat162float(row[label]) : lse;
    loss[r] = lse - target;
    if (lse_out != nullptr) lse_out[r] = lse;
  }
  __syncthreads();  // the label logit is read before gradients overwrite the row
  const float inv_s = 1.f / s;
  for (int i = threadIdx.x * 8; i < V; i += kCeThreads * 8) {
    float f[8];
    ld8(row + i, f);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float g = __expf(f[e] - m) * inv_s;
      if (i + e == label) g -= 1.f;
      f[e] = g * wgt;
    }
    st8(row + i, f);
  }
}

// ------------------------------------------------------------------ optimizer
__global__ void sumsq_kernel(const float* __restrict__ g, long n, float* __restrict__ out) {
  float acc = 0.f;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float v = g[i];
    acc += v * v;
  }
  acc = warp_sum(acc);
  __shared__ float red[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  if (warp == 0) {
    acc = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
    acc = warp_sum(acc);
    if (lane == 0) atomicAdd(out, acc);
  }
}

// AdamW with the clip coefficient derived on the device from the all-reduced
// squared norm, so the step needs no host synchronisation. A non-finite norm
// leaves every state untouched.
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ p_bf16, long n,
                             const float* __restrict__ sumsq, float max_norm, float lr, float b1, float b2, float eps,
                             float wd, float bc1, float bc2) {
  const float ss = *sumsq;
  if (!isfinite(ss)) return;
  float coef = 1.f;
  if (max_norm > 0.f) coef = fminf(1.f, max_norm / (sqrtf(ss) + 1e-6f));
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float gi = g[i] * coef;
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    float pi = p[i];
    pi -= lr * ((mi / bc1) / (sqrtf(vi / bc2) + eps) + wd * pi);
    p[i] = pi;
    if (p_bf16 != nullptr) p_bf16[i] = __float2bfloat16(pi);
  }
}

int sm_count(int dev) {
  int n = 0;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  return n;
}

}  // namespace

void rope_inplace(at::Tensor& x, const at::Tensor& pos, int64_t heads, int64_t d, double base, bool inverse) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.stride(-1) == 1, "rope: bf16 CUDA rows");
  TORCH_CHECK(pos.scalar_type() == at::kInt && pos.numel() == x.size(0), "rope: int32 positions [T]");
  TORCH_CHECK(d % 16 == 0, "rope: head dim multiple of 16");
  TORCH_CHECK(x.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0, "rope: aligned rows");
  const c10::cuda::CUDAGuard guard(x.device());
  const int T = x.size(0);
  const long total = (long)T * heads * (d / 16);
  if (total == 0) return;
  rope_kernel<<<(total + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), x.stride(0), pos.data_ptr<int>(), T, (int)heads, (int)d,
      (float)std::log2(base), inverse ? -1.f : 1.f);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

at::Tensor conv1d_silu_fwd(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& halo,
                           const at::Tensor& cu) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1, "conv: bf16 rows");
  const int T = x.size(0), C = x.size(1);
  TORCH_CHECK(w.size(0) == C && w.size(1) == kConvK && w.is_contiguous(), "conv: weight [C,4]");
  TORCH_CHECK(cu.scalar_type() == at::kInt, "conv: int32 cu_seqlens");
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor y = at::empty({T, C}, x.options());
  if (T == 0) return y;
  const __nv_bfloat16* hp = nullptr;
  if (halo) {
    TORCH_CHECK(halo->size(0) == kConvK - 1 && halo->size(1) == C && halo->is_contiguous(), "conv: halo [3,C]");
    hp = reinterpret_cast<const __nv_bfloat16*>(halo->data_ptr());
  }
  const bool vec = C % 8 == 0 && x.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(w.data_ptr()) & 15) == 0;
  if (vec && kConvTokenParallel) {
    dim3 gp((T + kConvTokP - 1) / kConvTokP, (C / 8 + 31) / 32);
    conv_fwd_tok_kernel<<<gp, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), hp, cu.data_ptr<int>(), (int)cu.numel() - 1, T, C,
        reinterpret_cast<__nv_bfloat16*>(y.data_ptr()));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return y;
  }
  if (vec) {
    dim3 gv((T + kConvTokV - 1) / kConvTokV, (C / 8 + 127) / 128);
    conv_fwd_vec_kernel<<<gv, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), hp, cu.data_ptr<int>(), (int)cu.numel() - 1, T, C,
        reinterpret_cast<__nv_bfloat16*>(y.data_ptr()));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return y;
  }
  dim3 grid((T + kConvTok - 1) / kConvTok, (C + 127) / 128);
  conv_fwd_kernel<<<grid, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), hp, cu.data_ptr<int>(), (int)cu.numel() - 1, T, C,
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y;
}

// Returns (dw fp32 [C,4], dhalo fp32 [3,C] or empty). dx written into `dx` (may be a strided view).
std::vector<at::Tensor> conv1d_silu_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                        const c10::optional<at::Tensor>& halo, const at::Tensor& cu, at::Tensor& dx) {
  const int T = x.size(0), C = x.size(1);
  TORCH_CHECK(dy.is_contiguous() && dy.size(0) == T && dy.size(1) == C, "conv bwd: dy [T,C] contiguous");
  TORCH_CHECK(dx.stride(1) == 1 && dx.size(0) == T && dx.size(1) == C, "conv bwd: dx rows");
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor dw = at::zeros({C, kConvK}, x.options().dtype(at::kFloat));
  at::Tensor dh;
  const __nv_bfloat16* hp = nullptr;
  float* dhp = nullptr;
  if (halo) {
    hp = reinterpret_cast<const __nv_bfloat16*>(halo->data_ptr());
    dh = at::zeros({kConvK - 1, C}, x.options().dtype(at::kFloat));
    dhp = dh.data_ptr<float>();
  }
  const bool vec = C % 8 == 0 && x.stride(0) % 8 == 0 && dx.stride(0) % 8 == 0 &&
                   (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(dx.data_ptr()) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(dy.data_ptr()) & 15) == 0;
  if (T > 0 && vec) {
    dim3 gv((T + kConvTokV - 1) / kConvTokV, (C / 8 + 127) / 128);
    conv_bwd_vec_kernel<<<gv, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
        x.stride(0), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), hp, cu.data_ptr<int>(),
        (int)cu.numel() - 1, T, C, reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), dx.stride(0),
        dw.data_ptr<float>(), dhp);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  } else if (T > 0) {
    dim3 grid((T + kConvTok - 1) / kConvTok, (C + 127) / 128);
    conv_bwd_kernel<<<grid, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
        x.stride(0), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), hp, cu.data_ptr<int>(),
        (int)cu.numel() - 1, T, C, reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), dx.stride(0),
        dw.data_ptr<float>(), dhp);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  if (halo) return {dw, dh};
  return {dw};
}

void swiglu_fwd(const at::Tensor& x, at::Tensor& y) {
  const int T = x.size(0), F = x.size(1) / 2;
  TORCH_CHECK(F % 8 == 0 && x.stride(1) == 1 && y.stride(1) == 1, "swiglu: F multiple of 8, unit stride");
  TORCH_CHECK(x.stride(0) % 8 == 0 && y.stride(0) % 8 == 0, "swiglu: row strides multiple of 8");
  const c10::cuda::CUDAGuard guard(x.device());
  const long total = (long)T * (F / 8);
  if (total == 0) return;
  swiglu_fwd_kernel<<<(total + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), y.stride(0), T, F);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void swiglu_bwd(const at::Tensor& dy, const at::Tensor& x, at::Tensor& dx) {
  const int T = x.size(0), F = x.size(1) / 2;
  const c10::cuda::CUDAGuard guard(x.device());
  const long total = (long)T * (F / 8);
  if (total == 0) return;
  swiglu_bwd_kernel<<<(total + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), dy.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
      reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), dx.stride(0), T, F);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ce_fused(at::Tensor& logits, const at::Tensor& labels, const at::Tensor& weight, at::Tensor& loss,
              const c10::optional<at::Tensor>& lse) {
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1, "ce: bf16 logits rows");
  TORCH_CHECK(labels.scalar_type() == at::kLong && weight.scalar_type() == at::kFloat, "ce: int64 labels, fp32 w");
  const int R = logits.size(0), V = logits.size(1);
  TORCH_CHECK(V % 8 == 0 && logits.stride(0) % 8 == 0, "ce: vocab and row stride multiples of 8");
  const c10::cuda::CUDAGuard guard(logits.device());
  if (R == 0) return;
  ce_fused_kernel<<<R, kCeThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), logits.stride(0), labels.data_ptr<int64_t>(),
      weight.data_ptr<float>(), V, loss.data_ptr<float>(), lse ? lse->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void sumsq_accumulate(const at::Tensor& g, at::Tensor& out) {
  TORCH_CHECK(g.scalar_type() == at::kFloat && g.is_contiguous() && out.scalar_type() == at::kFloat, "sumsq: fp32");
  const c10::cuda::CUDAGuard guard(g.device());
  const long n = g.numel();
  if (n == 0) return;
  const int blocks = std::min<long>((n + 1023) / 1024, sm_count(g.get_device()) * 4);
  sumsq_kernel<<<blocks, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(g.data_ptr<float>(), n, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adamw_step(at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v,
                const c10::optional<at::Tensor>& p_bf16, const at::Tensor& sumsq, double max_norm, double lr,
                double b1, double b2, double eps, double wd, double bc1, double bc2) {
  TORCH_CHECK(p.is_contiguous() && g.is_contiguous() && m.is_contiguous() && v.is_contiguous(), "adamw: flat");
  const c10::cuda::CUDAGuard guard(p.device());
  const long n = p.numel();
  if (n == 0) return;
  const int blocks = std::min<long>((n + 511) / 512, sm_count(p.get_device()) * 8);
  adamw_kernel<<<blocks, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
      p_bf16 ? reinterpret_cast<__nv_bfloat16*>(p_bf16->data_ptr()) : nullptr, n, sumsq.data_ptr<float>(),
      (float)max_norm, (float)lr, (float)b1, (float)b2, (float)eps, (float)wd, (float)bc1, (float)bc2);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace prism
