// chunk_gated_delta_rule, per-step kernel (CUDA cores), any D in {16, 32, 64, 128}.
//
// The recurrence of the reference (_ref_forward, operators/chunk_gated_delta_rule.py:291-308):
//   r   = h_{t-1} k_t            (h is [D_v, D_k], fp32)
//   h_t = g_t h_{t-1} + beta_t (v_t - r) k_t^T
//   o_t = h_t q_t                (rounded to the input dtype)
// One CTA per (batch, head).  The fp32 state lives in registers: thread tid owns
// row tid / TPR and CPT consecutive columns; the two row dot products per step
// are reduced across the TPR threads of a row with shuffles.  q/k/v of step t+1
// are staged in shared memory (double buffer) while step t computes, so a step
// costs one block barrier.  This is the path for D <= 64 and an independent
// on-device cross-check of the chunked tensor-core kernel.
#include "common.cuh"

namespace fo {
namespace {

constexpr int kStepThreads = 256;

template <typename T, typename G, int D>
__global__ void __launch_bounds__(kStepThreads)
gdr_step_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                const G* __restrict__ beta, const G* __restrict__ g, const float* __restrict__ h0,
                T* __restrict__ o, float* __restrict__ hT, const int* __restrict__ only,
                int64_t L) {
  // with `only`, heads whose entry is 0 are left alone (recomputation of the
  // heads the tensor-core kernel marked)
  if (only && only[blockIdx.x] == 0) return;
  constexpr int TPR = kStepThreads / D;  // threads per state row
  constexpr int CPT = D / TPR;           // columns per thread
  __shared__ float s_k[2][D], s_q[2][D], s_v[2][D], s_bg[2][2];
  const int tid = threadIdx.x;
  const int row = tid / TPR;
  const int c0 = (tid % TPR) * CPT;
  const int64_t head = blockIdx.x;
  const T* qh = q + head * L * D;
  const T* kh = k + head * L * D;
  const T* vh = v + head * L * D;
  T* oh = o + head * L * D;

  float hs[CPT];
#pragma unroll
  for (int c = 0; c < CPT; ++c) hs[c] = h0 ? h0[head * D * D + row * D + c0 + c] : 0.f;

  auto stage = [&](int64_t t, int buf) {
    if (tid < D) {
      s_k[buf][tid] = to_f<T>(kh[t * D + tid]);
      s_q[buf][tid] = to_f<T>(qh[t * D + tid]);
      s_v[buf][tid] = to_f<T>(vh[t * D + tid]);
    }
    if (tid == 0) {
      s_bg[buf][0] = to_f<G>(beta[head * L + t]);
      s_bg[buf][1] = to_f<G>(g[head * L + t]);
    }
  };
  if (L > 0) stage(0, 0);
  for (int64_t t = 0; t < L; ++t) {
    const int b = (int)(t & 1);
    __syncthreads();
    if (t + 1 < L) stage(t + 1, b ^ 1);
    float r = 0.f;
#pragma unroll
    for (int c = 0; c < CPT; ++c) r = fmaf(hs[c], s_k[b][c0 + c], r);
#pragma unroll
    for (int off = TPR / 2; off > 0; off >>= 1) r += __shfl_xor_sync(0xffffffffu, r, off);
    const float bu = s_bg[b][0] * (s_v[b][row] - r);
    const float gt = s_bg[b][1];
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      hs[c] = fmaf(gt, hs[c], bu * s_k[b][c0 + c]);
      acc = fmaf(hs[c], s_q[b][c0 + c], acc);
    }
#pragma unroll
    for (int off = TPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if ((tid % TPR) == 0) oh[t * D + row] = from_f<T>(acc);
  }
  if (hT) {
#pragma unroll
    for (int c = 0; c < CPT; ++c) hT[head * D * D + row * D + c0 + c] = hs[c];
  }
}

template <typename T, typename G>
int launch_step(const void* q, const void* k, const void* v, const void* beta, const void* g,
                const float* h0, void* o, float* hT, const int* only, int64_t BH, int64_t L,
                int64_t D, cudaStream_t st) {
#define FO_STEP(DD)                                                                          \
  gdr_step_kernel<T, G, DD><<<(unsigned)BH, kStepThreads, 0, st>>>(                          \
      (const T*)q, (const T*)k, (const T*)v, (const G*)beta, (const G*)g, h0, (T*)o, hT, only, L)
  switch (D) {
    case 16: FO_STEP(16); break;
    case 32: FO_STEP(32); break;
    case 64: FO_STEP(64); break;
    case 128: FO_STEP(128); break;
    default:
      set_error("D=%lld not in supported set {16,32,64,128}", (long long)D);
      return FO_EUNSUPPORTED;
  }
#undef FO_STEP
  return check_launch("gdr_step_kernel");
}

template <typename T>
int step_gate_dispatch(int gate_dtype, const void* q, const void* k, const void* v,
                       const void* beta, const void* g, const float* h0, void* o, float* hT,
                       const int* only, int64_t BH, int64_t L, int64_t D, cudaStream_t st) {
  switch (gate_dtype) {
    case FO_F32: return launch_step<T, float>(q, k, v, beta, g, h0, o, hT, only, BH, L, D, st);
    case FO_F16: return launch_step<T, __half>(q, k, v, beta, g, h0, o, hT, only, BH, L, D, st);
    case FO_BF16:
      return launch_step<T, __nv_bfloat16>(q, k, v, beta, g, h0, o, hT, only, BH, L, D, st);
  }
  set_error("chunk_gated_delta_rule: unsupported gate dtype code %d", gate_dtype);
  return FO_EDTYPE;
}

}  // namespace

int gdr_stepwise(const void* q, const void* k, const void* v, const void* beta, const void* g,
                 const float* h0, void* o, float* hT, int64_t B, int64_t H, int64_t L, int64_t D,
                 int dtype, int gate_dtype, cudaStream_t st, const int* only) {
  const int64_t BH = B * H;
  switch (dtype) {
    case FO_F32:
      return step_gate_dispatch<float>(gate_dtype, q, k, v, beta, g, h0, o, hT, only, BH, L, D, st);
    case FO_F16:
      return step_gate_dispatch<__half>(gate_dtype, q, k, v, beta, g, h0, o, hT, only, BH, L, D,
                                        st);
    case FO_BF16:
      return step_gate_dispatch<__nv_bfloat16>(gate_dtype, q, k, v, beta, g, h0, o, hT, only, BH,
                                               L, D, st);
  }
  set_error("chunk_gated_delta_rule: unsupported dtype code %d", dtype);
  return FO_EDTYPE;
}

}  // namespace fo

extern "C" int fo_gdr_fwd_stepwise(const void* q, const void* k, const void* v, const void* beta,
                                   const void* g, const float* h0, void* o, float* hT, int64_t B,
                                   int64_t H, int64_t L, int64_t D, int dtype, int gate_dtype,
                                   void* stream) {
  fo::clear_error();
  FO_CHECK_ARG(B >= 0 && H >= 0 && L >= 0, "chunk_gated_delta_rule: negative size");
  if (B * H == 0) return FO_OK;
  if (L == 0) {
    // no tokens: the final state is the initial one (the empty q, k, v, o may
    // have null data pointers)
    cudaError_t e = cudaSuccess;
    if (hT && h0)
      e = cudaMemcpyAsync(hT, h0, B * H * D * D * sizeof(float), cudaMemcpyDeviceToDevice,
                          fo::as_stream(stream));
    else if (hT)
      e = cudaMemsetAsync(hT, 0, B * H * D * D * sizeof(float), fo::as_stream(stream));
    if (e != cudaSuccess) {
      fo::set_error("chunk_gated_delta_rule: %s", cudaGetErrorString(e));
      return FO_ECUDA;
    }
    return FO_OK;
  }
  FO_CHECK_ARG(q && k && v && beta && g && o, "chunk_gated_delta_rule: null pointer");
  return fo::gdr_stepwise(q, k, v, beta, g, h0, o, hT, B, H, L, D, dtype, gate_dtype,
                          fo::as_stream(stream), nullptr);
}
