// Sequential inter-chunk state pass of the chunked gated delta rule (sm_100a).
//
// With the WY form of a chunk c (C = 64 tokens, per head):
//   Delta_c = U_c - W_c S_c                 [C, dv]
//   S_{c+1} = gamma_c S_c + Kd_c^T Delta_c  [dk, dv]
// where W = T(beta*exp(G)*K), U = T(beta*V), Kd = exp(G_last - G)*K, gamma =
// exp(G_last) and T = (I + L)^-1 (see ops/gdn.py). The forward kernel walks the
// chunks of one sequence and writes Delta, the state at every chunk start and
// the final state. The backward kernel walks them in reverse with
//   dDelta_c = dDelta_ext_c + Kd_c G
//   G       <- dS_ext_c + gamma_c G - W_c^T dDelta_c      (G = dL/dS_{c+1})
// and stores dDelta and G_{c+1} per chunk; the remaining gradients (dW, dKd,
// dgamma) are independent per chunk and computed as batched products outside.
// One CTA owns (sequence, head, 32-column slice of dv); the fp32 state slice
// stays in shared memory for the whole sequence.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace prism {
namespace gdn {

constexpr int C = 64;
constexpr int DK = 128;
constexpr int SL = 32;  // dv slice per CTA
constexpr int THREADS = 256;

struct Args {
  const float* W;      // [Nc, H, C, DK]
  const float* U;      // [Nc, H, C, DV]   (bwd: dDelta_ext)
  const float* Kd;     // [Nc, H, C, DK]
  const float* gamma;  // [Nc, H]
  const float* S_ext;  // fwd: S0 [nseq, H, DK, DV] (nullable); bwd: dS_ext [Nc, H, DK, DV]
  const float* S_end;  // bwd: dS_final [nseq, H, DK, DV] (nullable)
  const int* seq_chunks;  // [nseq+1]
  float* out_rows;     // fwd: Delta; bwd: dDelta   [Nc, H, C, DV]
  float* out_states;   // fwd: S_all; bwd: G_next   [Nc, H, DK, DV]
  float* out_final;    // fwd: S_final; bwd: dS0    [nseq, H, DK, DV]
  int H, DV;
};

// s_state[k][j] for k < DK, j < SL; rows of W/Kd in smem [C][DK]
__global__ void __launch_bounds__(THREADS) gdn_state_fwd_kernel(Args a) {
  extern __shared__ float sm[];
  float* sS = sm;                 // [DK][SL]
  float* sW = sS + DK * SL;       // [C][DK]
  float* sK = sW + C * DK;        // [C][DK]
  float* sD = sK + C * DK;        // [C][SL]
  const int seq = blockIdx.x, h = blockIdx.y, j0 = blockIdx.z * SL;
  const int t = threadIdx.x;
  const int H = a.H, DV = a.DV;
  const int c_begin = a.seq_chunks[seq], c_end = a.seq_chunks[seq + 1];
  for (int e = t; e < DK * SL; e += THREADS) {
    const int k = e / SL, j = e % SL;
    sS[e] = a.S_ext ? a.S_ext[(((long)seq * H + h) * DK + k) * DV + j0 + j] : 0.f;
  }
  const int jj = t % SL;
  const int grp = t / SL;  // 0..7
  for (int c = c_begin; c < c_end; ++c) {
    const long ch = (long)c * H + h;
    const float4* gW = reinterpret_cast<const float4*>(a.W + ch * C * DK);
    const float4* gK = reinterpret_cast<const float4*>(a.Kd + ch * C * DK);
    for (int e = t; e < C * DK / 4; e += THREADS) {
      reinterpret_cast<float4*>(sW)[e] = gW[e];
      reinterpret_cast<float4*>(sK)[e] = gK[e];
    }
    __syncthreads();  // also orders the previous chunk's state update
    // store S_c slice
    for (int e = t; e < DK * SL; e += THREADS) {
      const int k = e / SL, j = e % SL;
      a.out_states[(ch * DK + k) * DV + j0 + j] = sS[e];
    }
    // Delta[i][jj] = U - sum_k W[i][k] S[k][jj], rows i = grp*8 .. +7
    float acc[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) acc[r] = a.U[(ch * C + grp * 8 + r) * DV + j0 + jj];
#pragma unroll 4
    for (int k = 0; k < DK; ++k) {
      const float s = sS[k * SL + jj];
#pragma unroll
      for (int r = 0; r < 8; ++r) acc[r] -= sW[(grp * 8 + r) * DK + k] * s;
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      sD[(grp * 8 + r) * SL + jj] = acc[r];
      a.out_rows[(ch * C + grp * 8 + r) * DV + j0 + jj] = acc[r];
    }
    __syncthreads();
    // S[k][jj] = gamma S + sum_i Kd[i][k] Delta[i][jj], k = grp*16 .. +15
    const float gm = a.gamma[ch];
    float st[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) st[r] = gm * sS[(grp * 16 + r) * SL + jj];
#pragma unroll 4
    for (int i = 0; i < C; ++i) {
      const float d = sD[i * SL + jj];
#pragma unroll
      for (int r = 0; r < 16; ++r) st[r] += sK[i * DK + grp * 16 + r] * d;
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) sS[(grp * 16 + r) * SL + jj] = st[r];
    __syncthreads();
  }
  for (int e = t; e < DK * SL; e += THREADS) {
    const int k = e / SL, j = e % SL;
    a.out_final[(((long)seq * H + h) * DK + k) * DV + j0 + j] = sS[e];
  }
}

__global__ void __launch_bounds__(THREADS) gdn_state_bwd_kernel(Args a) {
  extern __shared__ float sm[];
  float* sG = sm;                 // [DK][SL]
  float* sW = sG + DK * SL;       // [C][DK]
  float* sK = sW + C * DK;        // [C][DK]
  float* sD = sK + C * DK;        // [C][SL]  dDelta
  const int seq = blockIdx.x, h = blockIdx.y, j0 = blockIdx.z * SL;
  const int t = threadIdx.x;
  const int H = a.H, DV = a.DV;
  const int c_begin = a.seq_chunks[seq], c_end = a.seq_chunks[seq + 1];
  for (int e = t; e < DK * SL; e += THREADS) {
    const int k = e / SL, j = e % SL;
    sG[e] = a.S_end ? a.S_end[(((long)seq * H + h) * DK + k) * DV + j0 + j] : 0.f;
  }
  const int jj = t % SL;
  const int grp = t / SL;
  for (int c = c_end - 1; c >= c_begin; --c) {
    const long ch = (long)c * H + h;
    const float4* gW = reinterpret_cast<const float4*>(a.W + ch * C * DK);
    const float4* gK = reinterpret_cast<const float4*>(a.Kd + ch * C * DK);
    for (int e = t; e < C * DK / 4; e += THREADS) {
      reinterpret_cast<float4*>(sW)[e] = gW[e];
      reinterpret_cast<float4*>(sK)[e] = gK[e];
    }
    __syncthreads();
    for (int e = t; e < DK * SL; e += THREADS) {
      const int k = e / SL, j = e % SL;
      a.out_states[(ch * DK + k) * DV + j0 + j] = sG[e];
    }
    // dDelta[i][jj] = dDelta_ext + sum_k Kd[i][k] G[k][jj]
    float acc[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) acc[r] = a.U[(ch * C + grp * 8 + r) * DV + j0 + jj];
#pragma unroll 4
    for (int k = 0; k < DK; ++k) {
      const float g = sG[k * SL + jj];
#pragma unroll
      for (int r = 0; r < 8; ++r) acc[r] += sK[(grp * 8 + r) * DK + k] * g;
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      sD[(grp * 8 + r) * SL + jj] = acc[r];
      a.out_rows[(ch * C + grp * 8 + r) * DV + j0 + jj] = acc[r];
    }
    __syncthreads();
    // G[k][jj] = dS_ext + gamma G - sum_i W[i][k] dDelta[i][jj]
    const float gm = a.gamma[ch];
    float gn[16];
#pragma unroll
    for (int r = 0; r < 16; ++r)
      gn[r] = a.S_ext[(ch * DK + grp * 16 + r) * DV + j0 + jj] + gm * sG[(grp * 16 + r) * SL + jj];
#pragma unroll 4
    for (int i = 0; i < C; ++i) {
      const float d = sD[i * SL + jj];
#pragma unroll
      for (int r = 0; r < 16; ++r) gn[r] -= sW[i * DK + grp * 16 + r] * d;
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) sG[(grp * 16 + r) * SL + jj] = gn[r];
    __syncthreads();
  }
  for (int e = t; e < DK * SL; e += THREADS) {
    const int k = e / SL, j = e % SL;
    a.out_final[(((long)seq * H + h) * DK + k) * DV + j0 + j] = sG[e];
  }
}

constexpr int SMEM = (DK * SL + 2 * C * DK + C * SL) * 4;

void check(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous(), "gdn_state: ", name,
              " must be contiguous fp32 CUDA");
}

}  // namespace gdn

// Returns nothing; all outputs preallocated.
void gdn_state_fwd(const at::Tensor& W, const at::Tensor& U, const at::Tensor& Kd, const at::Tensor& gamma,
                   const c10::optional<at::Tensor>& S0, const at::Tensor& seq_chunks, at::Tensor& Delta,
                   at::Tensor& S_all, at::Tensor& S_final) {
  using namespace gdn;
  check(W, "W");
  check(U, "U");
  check(Kd, "Kd");
  check(gamma, "gamma");
  TORCH_CHECK(W.size(2) == C && W.size(3) == DK, "gdn_state: chunk 64, key dim 128");
  const int H = W.size(1), DV = U.size(3);
  TORCH_CHECK(DV % SL == 0, "gdn_state: value dim must be a multiple of 32");
  const int nseq = seq_chunks.numel() - 1;
  const c10::cuda::CUDAGuard guard(W.device());
  static bool cfg = false;
  if (!cfg) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gdn_state_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    C10_CUDA_CHECK(cudaFuncSetAttribute(gdn_state_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    cfg = true;
  }
  Args a;
  a.W = W.data_ptr<float>();
  a.U = U.data_ptr<float>();
  a.Kd = Kd.data_ptr<float>();
  a.gamma = gamma.data_ptr<float>();
  a.S_ext = S0 ? S0->data_ptr<float>() : nullptr;
  a.S_end = nullptr;
  a.seq_chunks = seq_chunks.data_ptr<int>();
  a.out_rows = Delta.data_ptr<float>();
  a.out_states = S_all.data_ptr<float>();
  a.out_final = S_final.data_ptr<float>();
  a.H = H;
  a.DV = DV;
  if (nseq == 0) return;
  gdn_state_fwd_kernel<<<dim3(nseq, H, DV / SL), THREADS, SMEM, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gdn_state_bwd(const at::Tensor& W, const at::Tensor& dDelta_ext, const at::Tensor& Kd, const at::Tensor& gamma,
                   const at::Tensor& dS_ext, const c10::optional<at::Tensor>& dS_final, const at::Tensor& seq_chunks,
                   at::Tensor& dDelta, at::Tensor& G_next, at::Tensor& dS0) {
  using namespace gdn;
  check(W, "W");
  check(dDelta_ext, "dDelta_ext");
  check(dS_ext, "dS_ext");
  const int H = W.size(1), DV = dDelta_ext.size(3);
  const int nseq = seq_chunks.numel() - 1;
  const c10::cuda::CUDAGuard guard(W.device());
  Args a;
  a.W = W.data_ptr<float>();
  a.U = dDelta_ext.data_ptr<float>();
  a.Kd = Kd.data_ptr<float>();
  a.gamma = gamma.data_ptr<float>();
  a.S_ext = dS_ext.data_ptr<float>();
  a.S_end = dS_final ? dS_final->data_ptr<float>() : nullptr;
  a.seq_chunks = seq_chunks.data_ptr<int>();
  a.out_rows = dDelta.data_ptr<float>();
  a.out_states = G_next.data_ptr<float>();
  a.out_final = dS0.data_ptr<float>();
  a.H = H;
  a.DV = DV;
  if (nseq == 0) return;
  static bool cfg = false;
  if (!cfg) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gdn_state_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    cfg = true;
  }
  gdn_state_bwd_kernel<<<dim3(nseq, H, DV / SL), THREADS, SMEM, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace prism
