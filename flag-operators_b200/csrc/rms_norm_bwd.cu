// rms_norm backward (dx, dw) for sm_100a, consuming the inv_rms the forward
// returns.
//
// Semantics: the gradients of the reference CPU forward
// (operators/rms_norm.py:211-216), y = (x / rms) * w with
// rms = sqrt(mean(x^2) + eps) and inv = 1 / rms:
//   g  = dy * w
//   dx = inv * g - x * inv^3 * (sum_j g_j x_j) / N
//   dw = sum over rows of dy * x * inv
// in fp32, dx rounded once to x's dtype and dw to w's dtype.  The reference
// returns inv_rms for exactly this use (its forward is FlagGems-compatible); it
// ships no backward of its own.
//
// Design.  Vector path (16-byte aligned rows of up to 1024 vectors): persistent
// CTAs (one per SM, 512 threads) own whole rows and every thread the same VPT
// 16-byte column vectors of every row, so x and dy are read from HBM once, dx is
// written once, the row's dot product is one block reduction, and the thread's
// share of dw stays in registers across all the rows of its CTA.  The next
// row's x and dy are loaded before the current row's reduction (in flight
// during the barrier and the stores).  Each CTA writes its dw partial sums to a
// [CTAs, N] fp32 workspace and a column kernel adds them up in a fixed order
// (deterministic).  Measured slower: one vector per thread in 1024-thread CTAs.
// Generic path (any N, any alignment): a CTA per row with two passes over the
// row (the second from L2) for dx, and a row-chunked column kernel for dw.
#include "common.cuh"

namespace fo {
namespace {

constexpr int kBwdThreads = 512;
constexpr int kBwdRowChunks = 64;  // generic dw: row chunks (partial sums)

template <typename T, typename W, int VPT>
__global__ void __launch_bounds__(kBwdThreads, 1)
rms_bwd_vec_kernel(const T* __restrict__ dy, const T* __restrict__ x, const W* __restrict__ w,
                   const float* __restrict__ inv_rms, T* __restrict__ dx,
                   float* __restrict__ dw_part, int64_t M, int N) {
  constexpr int E = Vec16<T>::E;
  __shared__ float red[32];
  const int nvec = N / E;
  float wf[VPT][E];
  float dwa[VPT][E];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      wf[i][e] = v < nvec ? to_f<W>(w[(int64_t)v * E + e]) : 0.f;
      dwa[i][e] = 0.f;
    }
  }
  auto load = [&](int64_t row, uint4 (&ax)[VPT], uint4 (&ady)[VPT]) {
    const T* xr = x + row * (int64_t)N;
    const T* dr = dy + row * (int64_t)N;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int v = threadIdx.x + i * blockDim.x;
      ax[i] = v < nvec ? ld_global_stream_v4(xr + (int64_t)v * E) : make_uint4(0, 0, 0, 0);
      ady[i] = v < nvec ? ld_global_stream_v4(dr + (int64_t)v * E) : make_uint4(0, 0, 0, 0);
    }
  };
  uint4 cx[VPT], cdy[VPT];
  if (blockIdx.x < M) load(blockIdx.x, cx, cdy);
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    uint4 nx[VPT], ndy[VPT];
    if (row + gridDim.x < M) load(row + gridDim.x, nx, ndy);
    const float inv = inv_rms[row];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float fx[E], fd[E];
      unpack16<T>(cx[i], fx);
      unpack16<T>(cdy[i], fd);
#pragma unroll
      for (int e = 0; e < E; ++e) s = fmaf(fd[e] * wf[i][e], fx[e], s);
    }
    s = block_sum(s, red);
    const float c = inv * inv * inv * s / (float)N;
    T* dxr = dx + row * (int64_t)N;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int v = threadIdx.x + i * blockDim.x;
      if (v < nvec) {
        float fx[E], fd[E], o[E];
        unpack16<T>(cx[i], fx);
        unpack16<T>(cdy[i], fd);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          o[e] = fmaf(inv, fd[e] * wf[i][e], -c * fx[e]);
          dwa[i][e] = fmaf(fd[e] * fx[e], inv, dwa[i][e]);
        }
        st_global_stream_v4(dxr + (int64_t)v * E, pack16<T>(o));
      }
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      cx[i] = nx[i];
      cdy[i] = ndy[i];
    }
  }
  float* part = dw_part + (int64_t)blockIdx.x * N;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < nvec) {
#pragma unroll
      for (int e = 0; e < E; e += 4)
        *reinterpret_cast<float4*>(part + (int64_t)v * E + e) =
            make_float4(dwa[i][e], dwa[i][e + 1], dwa[i][e + 2], dwa[i][e + 3]);
    }
  }
}

// dx for any N / alignment: two passes over the row (the second hits L2).
template <typename T, typename W>
__global__ void __launch_bounds__(256)
rms_bwd_generic_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                       const W* __restrict__ w, const float* __restrict__ inv_rms,
                       T* __restrict__ dx, int64_t M, int64_t N) {
  __shared__ float red[32];
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const T* xr = x + row * N;
    const T* dr = dy + row * N;
    const float inv = inv_rms[row];
    float s = 0.f;
    for (int64_t j = threadIdx.x; j < N; j += blockDim.x)
      s = fmaf(to_f<T>(dr[j]) * to_f<W>(w[j]), to_f<T>(xr[j]), s);
    s = block_sum(s, red);
    const float c = inv * inv * inv * s / (float)N;
    T* dxr = dx + row * N;
    for (int64_t j = threadIdx.x; j < N; j += blockDim.x)
      dxr[j] = from_f<T>(fmaf(inv, to_f<T>(dr[j]) * to_f<W>(w[j]), -c * to_f<T>(xr[j])));
  }
}

// dw partial sums for any N: chunk r of the rows, one column per thread.
template <typename T>
__global__ void __launch_bounds__(256)
rms_dw_chunk_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                    const float* __restrict__ inv_rms, float* __restrict__ dw_part, int64_t M,
                    int64_t N) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= N) return;
  const int64_t rows = (M + gridDim.y - 1) / gridDim.y;
  const int64_t r0 = (int64_t)blockIdx.y * rows;
  const int64_t r1 = (r0 + rows < M) ? r0 + rows : M;
  float a = 0.f;
  for (int64_t r = r0; r < r1; ++r)
    a = fmaf(to_f<T>(dy[r * N + j]) * to_f<T>(x[r * N + j]), inv_rms[r], a);
  dw_part[(int64_t)blockIdx.y * N + j] = a;
}

// dw[j] = sum over the G partial rows.  A CTA owns 32 columns: warp q of 32
// adds rows q, q + 32, ... (lane = column, 128-byte coalesced rows; ~5 rows per
// warp for one CTA per SM, so each chain of dependent adds is short), then warp
// 0 adds the 32 warp sums in order, so the result does not depend on
// scheduling.
constexpr int kDwWarps = 32;
template <typename W>
__global__ void __launch_bounds__(32 * kDwWarps)
rms_dw_reduce_kernel(const float* __restrict__ dw_part, int G, int64_t N, W* __restrict__ dw) {
  __shared__ float acc[kDwWarps][33];
  const int lane = threadIdx.x & 31, q = threadIdx.x >> 5;
  const int64_t j = (int64_t)blockIdx.x * 32 + lane;
  float a = 0.f;
  if (j < N)
    for (int g = q; g < G; g += kDwWarps) a += dw_part[(int64_t)g * N + j];
  acc[q][lane] = a;
  __syncthreads();
  if (q == 0 && j < N) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < kDwWarps; ++k) t += acc[k][lane];
    dw[j] = from_f<W>(t);
  }
}

inline size_t round256(size_t b) { return (b + 255) & ~(size_t)255; }

// CTAs of the vector path (one per SM) and partial rows of the workspace.
int64_t vec_ctas(int64_t M) {
  const int64_t g = num_sms();
  return g < M ? g : (M > 0 ? M : 1);
}

template <typename T>
bool vec_path(const void* dy, const void* x, const void* dx, int64_t N) {
  constexpr int E = Vec16<T>::E;
  return aligned16(dy) && aligned16(x) && aligned16(dx) && N % E == 0 &&
         N / E <= (int64_t)kBwdThreads * 2;
}

template <typename T, typename W>
int run_bwd(const void* dy, const void* x, const void* w, const float* inv, void* dx, void* dw,
            int64_t M, int64_t N, void* ws, cudaStream_t st) {
  constexpr int E = Vec16<T>::E;
  float* part = reinterpret_cast<float*>(ws);
  int G;
  if (vec_path<T>(dy, x, dx, N)) {
    const int nvec = (int)(N / E);
    G = (int)vec_ctas(M);
    int threads = nvec <= kBwdThreads ? ((nvec + 31) / 32) * 32 : kBwdThreads;
    if (threads < 32) threads = 32;
    if (nvec <= threads)
      rms_bwd_vec_kernel<T, W, 1><<<G, threads, 0, st>>>((const T*)dy, (const T*)x, (const W*)w,
                                                          inv, (T*)dx, part, M, (int)N);
    else
      rms_bwd_vec_kernel<T, W, 2><<<G, threads, 0, st>>>((const T*)dy, (const T*)x, (const W*)w,
                                                          inv, (T*)dx, part, M, (int)N);
    if (int rc = check_launch("rms_bwd_vec_kernel")) return rc;
  } else {
    int64_t grid = (int64_t)num_sms() * 8;
    if (grid > M) grid = M;
    rms_bwd_generic_kernel<T, W><<<(unsigned)grid, 256, 0, st>>>(
        (const T*)dy, (const T*)x, (const W*)w, inv, (T*)dx, M, N);
    if (int rc = check_launch("rms_bwd_generic_kernel")) return rc;
    G = (int)(M < kBwdRowChunks ? M : kBwdRowChunks);
    dim3 gc((unsigned)((N + 255) / 256), (unsigned)G);
    rms_dw_chunk_kernel<T><<<gc, 256, 0, st>>>((const T*)dy, (const T*)x, inv, part, M, N);
    if (int rc = check_launch("rms_dw_chunk_kernel")) return rc;
  }
  rms_dw_reduce_kernel<W><<<(unsigned)((N + 31) / 32), 32 * kDwWarps, 0, st>>>(part, G, N, (W*)dw);
  return check_launch("rms_dw_reduce_kernel");
}

template <typename T>
int bwd_w(int w_dtype, const void* dy, const void* x, const void* w, const float* inv, void* dx,
          void* dw, int64_t M, int64_t N, void* ws, cudaStream_t st) {
  switch (w_dtype) {
    case FO_F32: return run_bwd<T, float>(dy, x, w, inv, dx, dw, M, N, ws, st);
    case FO_F16: return run_bwd<T, __half>(dy, x, w, inv, dx, dw, M, N, ws, st);
    case FO_BF16: return run_bwd<T, __nv_bfloat16>(dy, x, w, inv, dx, dw, M, N, ws, st);
  }
  set_error("rms_norm backward: unsupported weight dtype code %d", w_dtype);
  return FO_EDTYPE;
}

}  // namespace
}  // namespace fo

using namespace fo;

extern "C" int fo_rms_norm_bwd_workspace_bytes(int64_t M, int64_t N, int64_t* bytes) {
  clear_error();
  FO_CHECK_ARG(bytes && M >= 0 && N >= 0, "fo_rms_norm_bwd_workspace_bytes: bad argument");
  int64_t rows = vec_ctas(M);
  if (rows < kBwdRowChunks) rows = kBwdRowChunks;
  *bytes = (int64_t)round256((size_t)rows * (size_t)N * sizeof(float));
  return FO_OK;
}

extern "C" int fo_rms_norm_bwd(const void* dy, const void* x, const void* weight,
                               const float* inv_rms, void* dx, void* dw, int64_t M, int64_t N,
                               int x_dtype, int w_dtype, void* workspace, int64_t ws_bytes,
                               void* stream) {
  clear_error();
  FO_CHECK_ARG(M >= 0 && N > 0, "rms_norm backward: bad size M=%lld N=%lld", (long long)M,
               (long long)N);
  FO_CHECK_ARG(weight && dw, "rms_norm backward: null weight / dw pointer");
  cudaStream_t st = as_stream(stream);
  if (M == 0) {
    // no rows: dw is zero
    const size_t wb = (size_t)N * (w_dtype == FO_F32 ? 4 : 2);
    cudaMemsetAsync(dw, 0, wb, st);
    return check_launch("rms_norm backward (empty)");
  }
  FO_CHECK_ARG(dy && x && inv_rms && dx, "rms_norm backward: null pointer");
  int64_t need = 0;
  fo_rms_norm_bwd_workspace_bytes(M, N, &need);
  if (!workspace || ws_bytes < need) {
    set_error("rms_norm backward: workspace of %lld bytes required", (long long)need);
    return FO_EWORKSPACE;
  }
  switch (x_dtype) {
    case FO_F32: return bwd_w<float>(w_dtype, dy, x, weight, inv_rms, dx, dw, M, N, workspace, st);
    case FO_F16: return bwd_w<__half>(w_dtype, dy, x, weight, inv_rms, dx, dw, M, N, workspace, st);
    case FO_BF16:
      return bwd_w<__nv_bfloat16>(w_dtype, dy, x, weight, inv_rms, dx, dw, M, N, workspace, st);
  }
  set_error("rms_norm backward: unsupported input dtype code %d", x_dtype);
  return FO_EDTYPE;
}
