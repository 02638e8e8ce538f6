// rms_norm forward for sm_100a.
//
// Semantics follow the reference CPU branch, operators/rms_norm.py:209-216:
//   rms = sqrt(mean(x^2) + eps) in fp32;  y = x / rms * w (rounded once to x's
//   dtype);  inv_rms = 1 / rms.
// Here y = x * (1/rms) * w: the product differs from the quotient by at most
// one fp32 ulp before the final rounding.
//
// Design: a row is read from HBM exactly once.  A CTA owns whole rows; every
// thread keeps VPT 16-byte vectors of the row in registers (VPT = 2 and 512
// threads for rows of 16 KiB), the row's sum of squares is a block reduction,
// then the same registers are scaled and stored.  CTAs are persistent over rows
// (grid-stride), so the weight slice each thread needs is loaded into registers
// once per CTA, not once per row.
#include "common.cuh"

namespace fo {
namespace {

template <typename T, typename W, int VPT>
__global__ void __launch_bounds__(512, VPT <= 2 ? 2 : 1)
rms_fwd_vec_kernel(const T* __restrict__ x, const W* __restrict__ w, T* __restrict__ y,
                   float* __restrict__ inv_rms, int64_t M, int N, float eps) {
  constexpr int E = Vec16<T>::E;
  // The weight slice of a thread is cached packed (16 bytes of W per 16 bytes of
  // x when the dtypes match) and unpacked at use, keeping the register count low
  // enough for 4 CTAs of 512 threads per SM.
  constexpr int WB = E * (int)sizeof(W);        // weight bytes per x vector
  constexpr int WV = (WB + 15) / 16;            // 16-byte words per x vector
  __shared__ float red[32];
  const int nvec = N / E;

  uint4 wr[VPT][WV];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
#pragma unroll
    for (int u = 0; u < WV; ++u) {
      if (v < nvec && WB % 16 == 0) wr[i][u] = *reinterpret_cast<const uint4*>(
          reinterpret_cast<const uint8_t*>(w) + (int64_t)v * WB + u * 16);
      else wr[i][u] = make_uint4(0, 0, 0, 0);
    }
  }
  auto weight = [&](int i, int e, int v) -> float {
    if constexpr (WB % 16 == 0) {
      return to_f<W>(reinterpret_cast<const W*>(&wr[i][0])[e]);
    } else {
      return to_f<W>(w[(int64_t)v * E + e]);
    }
  };

  // The next row's loads are issued before this row's block reduction, so they
  // are in flight while the CTA waits at the barrier and stores (rows of up to
  // 4 vectors per thread; longer rows have no registers to spare for it).
  auto load_row = [&](int64_t row, uint4 (&dst)[VPT]) {
    const T* xr = x + row * (int64_t)N;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int v = threadIdx.x + i * blockDim.x;
      if (v < nvec) dst[i] = ld_global_stream_v4(xr + (int64_t)v * E);
      else dst[i] = make_uint4(0, 0, 0, 0);
    }
  };
  uint4 raw[VPT];
  if (blockIdx.x < M) load_row(blockIdx.x, raw);
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    T* yr = y + row * (int64_t)N;
    constexpr bool kPrefetch = VPT <= 4;
    uint4 nxt[VPT];
    if (kPrefetch && row + gridDim.x < M) load_row(row + gridDim.x, nxt);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float f[E];
      unpack16<T>(raw[i], f);
#pragma unroll
      for (int e = 0; e < E; ++e) ss = fmaf(f[e], f[e], ss);
    }
    ss = block_sum(ss, red);
    const float rms = sqrtf(ss / (float)N + eps);
    const float inv = 1.0f / rms;
    if (threadIdx.x == 0) inv_rms[row] = inv;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int v = threadIdx.x + i * blockDim.x;
      if (v < nvec) {
        float f[E];
        unpack16<T>(raw[i], f);
#pragma unroll
        for (int e = 0; e < E; ++e) f[e] = (f[e] * inv) * weight(i, e, v);
        st_global_stream_v4(yr + (int64_t)v * E, pack16<T>(f));
      }
    }
    if (kPrefetch) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) raw[i] = nxt[i];
    } else if (row + gridDim.x < M) {
      load_row(row + gridDim.x, raw);
    }
  }
}

// Any N / alignment: two passes over the row (the second one hits L2).
template <typename T, typename W>
__global__ void __launch_bounds__(256)
rms_fwd_generic_kernel(const T* __restrict__ x, const W* __restrict__ w, T* __restrict__ y,
                       float* __restrict__ inv_rms, int64_t M, int64_t N, float eps) {
  __shared__ float red[32];
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const T* xr = x + row * N;
    T* yr = y + row * N;
    float ss = 0.f;
    for (int64_t j = threadIdx.x; j < N; j += blockDim.x) {
      const float f = to_f<T>(xr[j]);
      ss = fmaf(f, f, ss);
    }
    ss = block_sum(ss, red);
    const float rms = sqrtf(ss / (float)N + eps);
    const float inv = 1.0f / rms;
    if (threadIdx.x == 0) inv_rms[row] = inv;
    for (int64_t j = threadIdx.x; j < N; j += blockDim.x)
      yr[j] = from_f<T>((to_f<T>(xr[j]) * inv) * to_f<W>(w[j]));
  }
}

template <typename T, typename W, int VPT>
int launch_vec(const void* x, const void* w, void* y, float* inv_rms, int64_t M, int N, float eps,
               cudaStream_t st) {
  constexpr int E = Vec16<T>::E;
  const int nvec = N / E;
  int threads = (nvec + VPT - 1) / VPT;
  threads = ((threads + 31) / 32) * 32;
  if (threads < 32) threads = 32;
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rms_fwd_vec_kernel<T, W, VPT>, threads, 0);
  if (per_sm < 1) per_sm = 1;
  int64_t grid = (int64_t)num_sms() * per_sm;
  if (grid > M) grid = M;
  rms_fwd_vec_kernel<T, W, VPT><<<(unsigned)grid, threads, 0, st>>>(
      (const T*)x, (const W*)w, (T*)y, inv_rms, M, N, eps);
  return check_launch("rms_fwd_vec_kernel");
}

template <typename T, typename W>
int launch(const void* x, const void* w, void* y, float* inv_rms, int64_t M, int64_t N, float eps,
           cudaStream_t st) {
  constexpr int E = Vec16<T>::E;
  const bool vec_ok = aligned16(x) && aligned16(y) && (N % E == 0) && N <= (int64_t)512 * 8 * E;
  if (vec_ok) {
    const int nvec = (int)(N / E);
    if (nvec <= 512) return launch_vec<T, W, 1>(x, w, y, inv_rms, M, (int)N, eps, st);
    if (nvec <= 1024) return launch_vec<T, W, 2>(x, w, y, inv_rms, M, (int)N, eps, st);
    if (nvec <= 2048) return launch_vec<T, W, 4>(x, w, y, inv_rms, M, (int)N, eps, st);
    return launch_vec<T, W, 8>(x, w, y, inv_rms, M, (int)N, eps, st);
  }
  int64_t grid = (int64_t)num_sms() * 8;
  if (grid > M) grid = M;
  rms_fwd_generic_kernel<T, W><<<(unsigned)grid, 256, 0, st>>>((const T*)x, (const W*)w, (T*)y,
                                                                inv_rms, M, N, eps);
  return check_launch("rms_fwd_generic_kernel");
}

template <typename T>
int dispatch_w(int w_dtype, const void* x, const void* w, void* y, float* inv_rms, int64_t M,
               int64_t N, float eps, cudaStream_t st) {
  switch (w_dtype) {
    case FO_F32: return launch<T, float>(x, w, y, inv_rms, M, N, eps, st);
    case FO_F16: return launch<T, __half>(x, w, y, inv_rms, M, N, eps, st);
    case FO_BF16: return launch<T, __nv_bfloat16>(x, w, y, inv_rms, M, N, eps, st);
  }
  set_error("rms_norm: unsupported weight dtype code %d", w_dtype);
  return FO_EDTYPE;
}

}  // namespace
}  // namespace fo

extern "C" int fo_rms_norm_fwd(const void* x, const void* weight, void* y, float* inv_rms,
                               int64_t M, int64_t N, float eps, int x_dtype, int w_dtype,
                               void* stream) {
  using namespace fo;
  clear_error();
  FO_CHECK_ARG(M >= 0 && N >= 0, "rms_norm: negative size M=%lld N=%lld", (long long)M,
               (long long)N);
  if (M == 0) return FO_OK;
  FO_CHECK_ARG(N > 0, "rms_norm: normalized size N must be > 0");
  FO_CHECK_ARG(x && weight && y && inv_rms, "rms_norm: null pointer");
  cudaStream_t st = as_stream(stream);
  switch (x_dtype) {
    case FO_F32: return dispatch_w<float>(w_dtype, x, weight, y, inv_rms, M, N, eps, st);
    case FO_F16: return dispatch_w<__half>(w_dtype, x, weight, y, inv_rms, M, N, eps, st);
    case FO_BF16: return dispatch_w<__nv_bfloat16>(w_dtype, x, weight, y, inv_rms, M, N, eps, st);
  }
  set_error("rms_norm: unsupported input dtype code %d", x_dtype);
  return FO_EDTYPE;
}
