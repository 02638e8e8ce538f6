// chunk_gated_delta_rule backward (CUDA cores, fp32), any D in {16, 32, 64, 128}.
//
// The reference ships no backward: its CPU branch (_ref_forward,
// operators/chunk_gated_delta_rule.py:286-310) is plain torch, so the gradients
// it defines are autograd's through the recurrence
//   h_t = g_t h_{t-1} + beta_t (v_t - h_{t-1} k_t) k_t^T ,   o_t = h_t q_t .
// With delta_t = v_t - h_{t-1} k_t and G the gradient with respect to h_t
// (do_t q_t^T plus what flows back from h_{t+1}), one step in reverse is
//   gk = G k_t;  dv_t = beta_t gk;  dbeta_t = gk . delta_t;  dg_t = <G, h_{t-1}>
//   dq_t = g_t h_{t-1}^T do_t + beta_t (delta_t . do_t) k_t        (= h_t^T do_t)
//   dk_t = beta_t (G^T delta_t - h_{t-1}^T gk)
//   G   <- g_t G - beta_t gk k_t^T                                (gradient wrt h_{t-1})
// and the initial state's gradient is the last G.
//
// The recurrence is separable by state row: row i of h and of G evolves on its
// own, and only dq, dk, dbeta and dg sum over rows.  One CTA per (batch, head),
// everything in fp32.  A thread holds two state rows (2p, 2p + 1) and D / 16 of
// their columns (s, s + 16, s + 32, ...; the 16 lanes of a row pair read 16
// consecutive floats of a staged k or q row: no shared-memory bank conflicts);
// a warp holds two row pairs.  So a row dot product is a 4-level shuffle over 16
// lanes, and a column sum over the warp's four rows is the thread's own two rows
// plus one shuffle (these shuffles and the staged-row loads share the MIO pipe,
// which bounds the step).
//   1. a forward pass over the sequence writes the state at every 16-step
//      checkpoint (workspace);
//   2. chunks in reverse: stage the chunk's q, k, v, do, beta, g in shared
//      memory, recompute its states from the checkpoint into a per-head scratch
//      (each thread reads back only what it wrote; 16 states of every head,
//      128 MB at 128 heads of D = 128, mostly stay in L2), then run the reverse
//      steps, each loading the next step's state as soon as the current one is
//      dead so that the load overlaps the barrier and the block sums.  The
//      column sums (dq, dk) and scalar sums (dbeta, dg) of a step go through a
//      double-buffered shared-memory block, one slot per warp, added over the
//      warps in a fixed order: one barrier per step, and the result does not
//      depend on scheduling.
// No waits other than block barriers.
#include "common.cuh"

namespace fo {
namespace {

constexpr int kBwdChunk = 16;  // steps between state checkpoints
constexpr int kBwdSeg = 16;    // lanes per row pair (column stride of a thread)

template <int D>
struct BwdCfg {
  static constexpr int CPT = D / kBwdSeg;    // columns per thread (of each of its two rows)
  static constexpr int NT = (D / 2) * kBwdSeg;  // threads per CTA (= 8 D)
  static constexpr int NW = NT / 32;         // warps
  static constexpr int RED = 2 * D + 4;      // floats per warp in a reduction buffer
};

template <int D>
constexpr size_t bwd_smem_bytes() {
  return sizeof(float) *
         (4 * (size_t)kBwdChunk * D + 2 * kBwdChunk + 2 * (size_t)BwdCfg<D>::NW * BwdCfg<D>::RED);
}

// N consecutive floats between registers and 8- or 16-byte aligned memory
template <int N>
__device__ __forceinline__ void ld_seg(const float* p, float* r) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
      const float4 x = reinterpret_cast<const float4*>(p)[i];
      r[4 * i] = x.x;
      r[4 * i + 1] = x.y;
      r[4 * i + 2] = x.z;
      r[4 * i + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
      const float2 x = reinterpret_cast<const float2*>(p)[i];
      r[2 * i] = x.x;
      r[2 * i + 1] = x.y;
    }
  }
}

template <int N>
__device__ __forceinline__ void st_seg(float* p, const float* r) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N / 4; ++i)
      reinterpret_cast<float4*>(p)[i] =
          make_float4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < N / 2; ++i)
      reinterpret_cast<float2*>(p)[i] = make_float2(r[2 * i], r[2 * i + 1]);
  }
}

// sum over the 16 lanes of a row pair
__device__ __forceinline__ float row_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  x += __shfl_xor_sync(0xffffffffu, x, 4);
  x += __shfl_xor_sync(0xffffffffu, x, 8);
  return x;
}

// sum over the warp's two row pairs (lanes with the same columns)
__device__ __forceinline__ float pair_sum(float x) {
  return x + __shfl_xor_sync(0xffffffffu, x, 16);
}

template <typename T, typename Gt, int D>
__global__ void __launch_bounds__(BwdCfg<D>::NT, 1)
gdr_bwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
               const Gt* __restrict__ beta, const Gt* __restrict__ g, const float* __restrict__ h0,
               const T* __restrict__ dout, const float* __restrict__ dhT, T* __restrict__ dq,
               T* __restrict__ dk, T* __restrict__ dv, Gt* __restrict__ dbeta,
               Gt* __restrict__ dg, float* __restrict__ dh0, float* __restrict__ ckpt,
               float* __restrict__ scratch, int64_t L) {
  using C = BwdCfg<D>;
  constexpr int CPT = C::CPT, NT = C::NT, NW = C::NW, RED = C::RED, CH = kBwdChunk;
  constexpr int S = kBwdSeg;
  extern __shared__ float bsm[];
  float* s_q = bsm;              // [CH][D] each, fp32
  float* s_k = s_q + CH * D;
  float* s_v = s_k + CH * D;
  float* s_do = s_v + CH * D;
  float* s_b = s_do + CH * D;    // [CH]
  float* s_g = s_b + CH;         // [CH]
  float* s_red = s_g + CH;       // [2][NW][RED]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int seg = tid % S;             // columns seg + S * c
  const int r0 = 2 * (tid / S);        // rows r0 and r0 + 1
  const int64_t head = blockIdx.x;
  const int64_t nch = (L + CH - 1) / CH;
  const int64_t chs = L < CH ? L : CH;  // scratch states per head
  const int64_t DD = (int64_t)D * D;
  const T* qh = q + head * L * D;
  const T* kh = k + head * L * D;
  const T* vh = v + head * L * D;
  const T* doh = dout + head * L * D;
  float* ck = ckpt + head * nch * DD;
  float* sc = scratch + head * chs * DD;
  // this thread's 2 * CPT values of a [D, D] state: in the workspace
  // (checkpoints, scratch) one contiguous segment, read back only by this
  // thread; in the caller's row-major h0, dhT and dh0 at (r0 + e) * D + seg + S c
  const int64_t my = (int64_t)tid * (2 * CPT);
  auto ld_cols = [&](const float* p, float (*r)[CPT]) {
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
      for (int c = 0; c < CPT; ++c) r[e][c] = p[(int64_t)(r0 + e) * D + seg + S * c];
  };

  // chunk c's inputs into shared memory as fp32; returns its step count
  auto stage = [&](int64_t c, bool full) {
    const int64_t t0 = c * CH;
    const int n = (int)((L - t0) < CH ? (L - t0) : CH);
    for (int i = tid; i < CH * D; i += NT) {
      const bool in = (i / D) < n;
      const int64_t gi = t0 * D + i;
      s_k[i] = in ? to_f<T>(kh[gi]) : 0.f;
      s_v[i] = in ? to_f<T>(vh[gi]) : 0.f;
      if (full) {
        s_q[i] = in ? to_f<T>(qh[gi]) : 0.f;
        s_do[i] = in ? to_f<T>(doh[gi]) : 0.f;
      }
    }
    if (tid < CH) {
      const bool in = tid < n;
      s_b[tid] = in ? to_f<Gt>(beta[head * L + t0 + tid]) : 0.f;
      s_g[tid] = in ? to_f<Gt>(g[head * L + t0 + tid]) : 1.f;
    }
    return n;
  };

  // one forward step of this thread's two row segments
  auto fwd_step = [&](float (*h)[CPT], int tl) {
    const float* kr = s_k + tl * D + seg;
    float kv[CPT];
#pragma unroll
    for (int c = 0; c < CPT; ++c) kv[c] = kr[S * c];
    float r[2] = {0.f, 0.f};
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      r[0] = fmaf(h[0][c], kv[c], r[0]);
      r[1] = fmaf(h[1][c], kv[c], r[1]);
    }
    r[0] = row_sum(r[0]);
    r[1] = row_sum(r[1]);
    const float bt = s_b[tl], gt = s_g[tl];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float bu = bt * (s_v[tl * D + r0 + e] - r[e]);
#pragma unroll
      for (int c = 0; c < CPT; ++c) h[e][c] = fmaf(gt, h[e][c], bu * kv[c]);
    }
  };

  // ---- 1. forward: the state entering every chunk
  {
    float h[2][CPT];
    if (h0) {
      ld_cols(h0 + head * DD, h);
    } else {
#pragma unroll
      for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int c = 0; c < CPT; ++c) h[e][c] = 0.f;
    }
    for (int64_t c = 0; c < nch; ++c) {
      __syncthreads();  // the previous chunk's staged rows are no longer read
      const int n = stage(c, false);
      __syncthreads();
      st_seg<2 * CPT>(ck + c * DD + my, &h[0][0]);
      for (int tl = 0; tl < n; ++tl) fwd_step(h, tl);
    }
  }

  // ---- 2. chunks in reverse
  float G[2][CPT];
  if (dhT) {
    ld_cols(dhT + head * DD, G);
  } else {
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
      for (int c = 0; c < CPT; ++c) G[e][c] = 0.f;
  }
  int rb = 0;
  for (int64_t c = nch - 1; c >= 0; --c) {
    __syncthreads();  // the last step's readers of the staged rows are done
    const int n = stage(c, true);
    __syncthreads();
    {
      // the chunk's states, recomputed from its checkpoint: scratch[tl] = the
      // state before step tl
      float h[2][CPT];
      ld_seg<2 * CPT>(ck + c * DD + my, &h[0][0]);
      for (int tl = 0; tl < n; ++tl) {
        st_seg<2 * CPT>(sc + tl * DD + my, &h[0][0]);
        fwd_step(h, tl);
      }
    }
    float hp[2][CPT];  // the state before step tl
    ld_seg<2 * CPT>(sc + (n - 1) * DD + my, &hp[0][0]);
    for (int tl = n - 1; tl >= 0; --tl) {
      const int64_t t = c * CH + tl;
      const float* kr = s_k + tl * D + seg;
      const float* qr = s_q + tl * D + seg;
      float kv[CPT], qv[CPT];
#pragma unroll
      for (int cc = 0; cc < CPT; ++cc) {
        kv[cc] = kr[S * cc];
        qv[cc] = qr[S * cc];
      }
      const float bt = s_b[tl], gt = s_g[tl];
      float do_r[2], gk[2], hk[2], gh[2], delta[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        do_r[e] = s_do[tl * D + r0 + e];
        gk[e] = 0.f;
        hk[e] = 0.f;
        gh[e] = 0.f;
#pragma unroll
        for (int cc = 0; cc < CPT; ++cc) {
          G[e][cc] = fmaf(do_r[e], qv[cc], G[e][cc]);
          gk[e] = fmaf(G[e][cc], kv[cc], gk[e]);
          hk[e] = fmaf(hp[e][cc], kv[cc], hk[e]);
          gh[e] = fmaf(G[e][cc], hp[e][cc], gh[e]);
        }
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        gk[e] = row_sum(gk[e]);
        hk[e] = row_sum(hk[e]);
        gh[e] = row_sum(gh[e]);
        delta[e] = s_v[tl * D + r0 + e] - hk[e];
      }
      if (seg == 0) {
        dv[(head * L + t) * D + r0] = from_f<T>(bt * gk[0]);
        dv[(head * L + t) * D + r0 + 1] = from_f<T>(bt * gk[1]);
      }
      float* red = s_red + (rb * NW + warp) * RED;
#pragma unroll
      for (int cc = 0; cc < CPT; ++cc) {
        const float pq = pair_sum(fmaf(do_r[0], hp[0][cc], do_r[1] * hp[1][cc]));
        const float pk = pair_sum(fmaf(G[0][cc], delta[0], -gk[0] * hp[0][cc]) +
                                  fmaf(G[1][cc], delta[1], -gk[1] * hp[1][cc]));
        if (lane < S) {
          red[seg + S * cc] = pq;
          red[D + seg + S * cc] = pk;
        }
      }
      // hp is dead from here on: the next step's state loads during the sums
      if (tl > 0) ld_seg<2 * CPT>(sc + (tl - 1) * DD + my, &hp[0][0]);
      const float s_gd = pair_sum(fmaf(gk[0], delta[0], gk[1] * delta[1]));
      const float s_gh = pair_sum(gh[0] + gh[1]);
      const float s_dd = pair_sum(fmaf(do_r[0], delta[0], do_r[1] * delta[1]));
      if (lane == 0) {
        red[2 * D] = s_gd;
        red[2 * D + 1] = s_gh;
        red[2 * D + 2] = s_dd;
      }
#pragma unroll
      for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int cc = 0; cc < CPT; ++cc) G[e][cc] = fmaf(gt, G[e][cc], -bt * gk[e] * kv[cc]);
      __syncthreads();
      // the step's sums over all rows, warps added in a fixed order
      const float* rr = s_red + rb * NW * RED;
      if (tid < D) {
        float sq = 0.f, sd = 0.f;
#pragma unroll 4
        for (int w = 0; w < NW; ++w) {
          sq += rr[w * RED + tid];
          sd += rr[w * RED + 2 * D + 2];
        }
        dq[(head * L + t) * D + tid] = from_f<T>(fmaf(gt, sq, bt * s_k[tl * D + tid] * sd));
      } else if (tid < 2 * D) {
        float sum = 0.f;
#pragma unroll 4
        for (int w = 0; w < NW; ++w) sum += rr[w * RED + tid];
        dk[(head * L + t) * D + (tid - D)] = from_f<T>(bt * sum);
      } else if (tid < 2 * D + 2) {
        const int which = tid - 2 * D;  // 0: dbeta, 1: dg
        float sum = 0.f;
#pragma unroll 4
        for (int w = 0; w < NW; ++w) sum += rr[w * RED + 2 * D + which];
        if (which == 0)
          dbeta[head * L + t] = from_f<Gt>(sum);
        else
          dg[head * L + t] = from_f<Gt>(sum);
      }
      rb ^= 1;
    }
  }
  if (dh0) {
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
      for (int c = 0; c < CPT; ++c) dh0[head * DD + (int64_t)(r0 + e) * D + seg + S * c] = G[e][c];
  }
}

template <typename T, typename Gt, int D>
int launch_bwd(const void* q, const void* k, const void* v, const void* beta, const void* g,
               const float* h0, const void* dout, const float* dhT, void* dq, void* dk, void* dv,
               void* dbeta, void* dg, float* dh0, float* ckpt, float* scratch, int64_t BH,
               int64_t L, cudaStream_t st) {
  auto kern = gdr_bwd_kernel<T, Gt, D>;
  constexpr size_t smem = bwd_smem_bytes<D>();
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess) {
    set_error("gdr_bwd_kernel: cannot reserve %zu bytes of shared memory", smem);
    return FO_ECUDA;
  }
  kern<<<(unsigned)BH, BwdCfg<D>::NT, smem, st>>>(
      (const T*)q, (const T*)k, (const T*)v, (const Gt*)beta, (const Gt*)g, h0, (const T*)dout,
      dhT, (T*)dq, (T*)dk, (T*)dv, (Gt*)dbeta, (Gt*)dg, dh0, ckpt, scratch, L);
  return check_launch("gdr_bwd_kernel");
}

template <typename T, typename Gt>
int bwd_dim_dispatch(int64_t D, const void* q, const void* k, const void* v, const void* beta,
                     const void* g, const float* h0, const void* dout, const float* dhT, void* dq,
                     void* dk, void* dv, void* dbeta, void* dg, float* dh0, float* ckpt,
                     float* scratch, int64_t BH, int64_t L, cudaStream_t st) {
#define FO_BWD(DD)                                                                            \
  return launch_bwd<T, Gt, DD>(q, k, v, beta, g, h0, dout, dhT, dq, dk, dv, dbeta, dg, dh0,   \
                               ckpt, scratch, BH, L, st)
  switch (D) {
    case 16: FO_BWD(16);
    case 32: FO_BWD(32);
    case 64: FO_BWD(64);
    case 128: FO_BWD(128);
  }
#undef FO_BWD
  set_error("D=%lld not in supported set {16,32,64,128}", (long long)D);
  return FO_EUNSUPPORTED;
}

template <typename T>
int bwd_gate_dispatch(int gate_dtype, int64_t D, const void* q, const void* k, const void* v,
                      const void* beta, const void* g, const float* h0, const void* dout,
                      const float* dhT, void* dq, void* dk, void* dv, void* dbeta, void* dg,
                      float* dh0, float* ckpt, float* scratch, int64_t BH, int64_t L,
                      cudaStream_t st) {
  switch (gate_dtype) {
    case FO_F32:
      return bwd_dim_dispatch<T, float>(D, q, k, v, beta, g, h0, dout, dhT, dq, dk, dv, dbeta, dg,
                                        dh0, ckpt, scratch, BH, L, st);
    case FO_F16:
      return bwd_dim_dispatch<T, __half>(D, q, k, v, beta, g, h0, dout, dhT, dq, dk, dv, dbeta,
                                         dg, dh0, ckpt, scratch, BH, L, st);
    case FO_BF16:
      return bwd_dim_dispatch<T, __nv_bfloat16>(D, q, k, v, beta, g, h0, dout, dhT, dq, dk, dv,
                                                dbeta, dg, dh0, ckpt, scratch, BH, L, st);
  }
  set_error("chunk_gated_delta_rule backward: unsupported gate dtype code %d", gate_dtype);
  return FO_EDTYPE;
}

bool bwd_dim_ok(int64_t D) { return D == 16 || D == 32 || D == 64 || D == 128; }

int bwd_bad_dim(int64_t D) {
  set_error("D=%lld not in supported set {16,32,64,128}", (long long)D);
  return FO_EUNSUPPORTED;
}

// checkpoints (one state per 16 steps) + one chunk of recomputed states, per head
int64_t bwd_workspace_floats(int64_t BH, int64_t L, int64_t D) {
  const int64_t nch = (L + kBwdChunk - 1) / kBwdChunk;
  const int64_t chs = L < kBwdChunk ? L : kBwdChunk;
  return BH * (nch + chs) * D * D;
}

}  // namespace
}  // namespace fo

extern "C" int fo_gdr_bwd_workspace_bytes(int64_t B, int64_t H, int64_t L, int64_t D,
                                          int64_t* bytes) {
  fo::clear_error();
  FO_CHECK_ARG(bytes, "chunk_gated_delta_rule backward: null pointer");
  FO_CHECK_ARG(B >= 0 && H >= 0 && L >= 0, "chunk_gated_delta_rule backward: negative size");
  if (!fo::bwd_dim_ok(D)) return fo::bwd_bad_dim(D);
  *bytes = fo::bwd_workspace_floats(B * H, L, D) * (int64_t)sizeof(float);
  return FO_OK;
}

extern "C" int fo_gdr_bwd(const void* q, const void* k, const void* v, const void* beta,
                          const void* g, const float* h0, const void* d_o, const float* dhT,
                          void* dq, void* dk, void* dv, void* dbeta, void* dg, float* dh0,
                          int64_t B, int64_t H, int64_t L, int64_t D, int dtype, int gate_dtype,
                          void* workspace, int64_t workspace_bytes, void* stream) {
  fo::clear_error();
  FO_CHECK_ARG(B >= 0 && H >= 0 && L >= 0, "chunk_gated_delta_rule backward: negative size");
  if (!fo::bwd_dim_ok(D)) return fo::bwd_bad_dim(D);
  const int64_t BH = B * H;
  if (BH == 0) return FO_OK;
  cudaStream_t st = fo::as_stream(stream);
  if (L == 0) {
    // no steps: the initial state's gradient is the final state's (the empty
    // sequence tensors may have null data pointers)
    cudaError_t e = cudaSuccess;
    if (dh0 && dhT)
      e = cudaMemcpyAsync(dh0, dhT, BH * D * D * sizeof(float), cudaMemcpyDeviceToDevice, st);
    else if (dh0)
      e = cudaMemsetAsync(dh0, 0, BH * D * D * sizeof(float), st);
    if (e != cudaSuccess) {
      fo::set_error("chunk_gated_delta_rule backward: %s", cudaGetErrorString(e));
      return FO_ECUDA;
    }
    return FO_OK;
  }
  FO_CHECK_ARG(q && k && v && beta && g && d_o && dq && dk && dv && dbeta && dg,
               "chunk_gated_delta_rule backward: null pointer");
  FO_CHECK_ARG(BH <= 0x7fffffffLL, "chunk_gated_delta_rule backward: too many heads");
  const int64_t need = fo::bwd_workspace_floats(BH, L, D) * (int64_t)sizeof(float);
  if (!workspace || workspace_bytes < need) {
    fo::set_error("chunk_gated_delta_rule backward: workspace of %lld bytes, needs %lld",
                  (long long)workspace_bytes, (long long)need);
    return FO_EWORKSPACE;
  }
  FO_CHECK_ARG(fo::aligned16(workspace),
               "chunk_gated_delta_rule backward: the workspace must be 16-byte aligned");
  float* ckpt = static_cast<float*>(workspace);
  const int64_t nch = (L + fo::kBwdChunk - 1) / fo::kBwdChunk;
  float* scratch = ckpt + BH * nch * D * D;
  switch (dtype) {
    case FO_F32:
      return fo::bwd_gate_dispatch<float>(gate_dtype, D, q, k, v, beta, g, h0, d_o, dhT, dq, dk,
                                          dv, dbeta, dg, dh0, ckpt, scratch, BH, L, st);
    case FO_F16:
      return fo::bwd_gate_dispatch<__half>(gate_dtype, D, q, k, v, beta, g, h0, d_o, dhT, dq, dk,
                                           dv, dbeta, dg, dh0, ckpt, scratch, BH, L, st);
    case FO_BF16:
      return fo::bwd_gate_dispatch<__nv_bfloat16>(gate_dtype, D, q, k, v, beta, g, h0, d_o, dhT,
                                                  dq, dk, dv, dbeta, dg, dh0, ckpt, scratch, BH,
                                                  L, st);
  }
  fo::set_error("chunk_gated_delta_rule backward: unsupported dtype code %d", dtype);
  return FO_EDTYPE;
}
