// Fused cross-entropy (forward, backward, vocabulary-sharded pieces) for sm_100a.
//
// Semantics follow the reference CPU branch, F.cross_entropy
// (operators/fused_cross_entropy.py:327-331), including label smoothing:
//   loss_b = lse_b - (1 - e) x[b, t_b] - e * mean_j x[b, j]   (0 when t_b == ignore_index)
//   dloss/dx[b, j] = scale_b * (softmax_j - (1 - e)[j == t_b] - e / V)
// with scale_b = dout (* 1/n_valid for 'mean').  'mean' over zero valid rows is
// 0/0 = NaN, as torch.
//
// Design: one CTA per row (grid-stride persistent).  Pass 1 streams the row once
// with 16-byte loads and keeps an online (max, sum exp) pair per thread, merged
// by a block reduction.  When the gradient is wanted in the same call, pass 2
// re-reads the row — pass 1 loaded it with an L2 evict_last policy so the second
// read is served from L2 — and writes dlogits, so forward+backward costs one
// HBM read and one HBM write of B x V.  exp is exp2 with a pre-scaled argument
// (one FFMA + one MUFU.EX2 per element).
#include <math.h>

#include "common.cuh"

namespace fo {
namespace {

constexpr int kThreads = 512;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// packed fp32x2 arithmetic: one instruction for two lanes (sm_100a)
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(r)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)),
        "l"(*reinterpret_cast<uint64_t*>(&c)));
  return *reinterpret_cast<float2*>(&r);
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;"
      : "=l"(r)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)));
  return *reinterpret_cast<float2*>(&r);
}

// Sum of E (even, >= 4) floats as a tree of packed additions.
template <int E>
__device__ __forceinline__ float sum_vec(const float* e) {
  float2 p[E / 2];
#pragma unroll
  for (int i = 0; i < E / 2; ++i) p[i] = make_float2(e[2 * i], e[2 * i + 1]);
#pragma unroll
  for (int w = 1; w < E / 2; w <<= 1)
#pragma unroll
    for (int i = 0; i + w < E / 2; i += 2 * w) p[i] = add2(p[i], p[i + w]);
  return p[0].x + p[0].y;
}

// Asks L2 for the 16-byte-aligned interior of [p, p + bytes) with bulk
// prefetches of at most 32 KiB, one per thread of the first warps: the whole row
// is requested from DRAM at once instead of as the threads' loads reach it.
__device__ __forceinline__ void l2_prefetch(const void* p, int64_t bytes) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uintptr_t a0 = (a + 15) & ~(uintptr_t)15;
  const uintptr_t a1 = (a + (uintptr_t)bytes) & ~(uintptr_t)15;
  if (a1 <= a0) return;
  constexpr uintptr_t kPiece = 32768;
  for (uintptr_t off = (uintptr_t)threadIdx.x * kPiece; a0 + off < a1; off += blockDim.x * kPiece) {
    const uintptr_t n = (a1 - a0 - off) < kPiece ? (a1 - a0 - off) : kPiece;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a0 + off), "r"((uint32_t)n)
                 : "memory");
  }
}

struct MS {
  float m;  // running max
  float s;  // sum of exp(x - m)
};

__device__ __forceinline__ MS ms_merge(MS a, MS b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return {m, 0.f};
  return {m, a.s * fast_exp2((a.m - m) * kLog2e) + b.s * fast_exp2((b.m - m) * kLog2e)};
}

template <int E>
__device__ __forceinline__ void ms_add_vec(MS& st, float& rsum, const float* f, bool ls) {
  float lm = f[0];
#pragma unroll
  for (int i = 1; i < E; ++i) lm = fmaxf(lm, f[i]);
  if (lm > st.m) {
    st.s = (st.m == -INFINITY) ? 0.f : st.s * fast_exp2((st.m - lm) * kLog2e);
    st.m = lm;
  }
  if (st.m != -INFINITY) {
    // arguments two at a time, tree sum of the vector, then one add into the
    // running sum (short dependency chain)
    const float mb = -st.m * kLog2e;
    const float2 l2 = make_float2(kLog2e, kLog2e), b2 = make_float2(mb, mb);
    float e[E];
#pragma unroll
    for (int i = 0; i < E; i += 2) {
      const float2 a = fma2(make_float2(f[i], f[i + 1]), l2, b2);
      e[i] = fast_exp2(a.x);
      e[i + 1] = fast_exp2(a.y);
    }
    st.s += sum_vec<E>(e);
  }
  if (ls) rsum += sum_vec<E>(f);
}

__device__ __forceinline__ void ms_add_scalar(MS& st, float& rsum, float f, bool ls) {
  if (f > st.m) {
    st.s = (st.m == -INFINITY) ? 0.f : st.s * fast_exp2((st.m - f) * kLog2e);
    st.m = f;
  }
  if (st.m != -INFINITY) st.s += fast_exp2((f - st.m) * kLog2e);
  if (ls) rsum += f;
}

// Block-wide merge of (m, s) and of the row sum; result valid in every thread.
__device__ __forceinline__ void block_ms(MS& st, float& rsum, float* sm) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MS other{__shfl_xor_sync(0xffffffffu, st.m, o), __shfl_xor_sync(0xffffffffu, st.s, o)};
    st = ms_merge(st, other);
    rsum += __shfl_xor_sync(0xffffffffu, rsum, o);
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) {
    sm[wid] = st.m;
    sm[32 + wid] = st.s;
    sm[64 + wid] = rsum;
  }
  __syncthreads();
  MS t{lane < nw ? sm[lane] : -INFINITY, lane < nw ? sm[32 + lane] : 0.f};
  float r = lane < nw ? sm[64 + lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MS other{__shfl_xor_sync(0xffffffffu, t.m, o), __shfl_xor_sync(0xffffffffu, t.s, o)};
    t = ms_merge(t, other);
    r += __shfl_xor_sync(0xffffffffu, r, o);
  }
  st = t;
  rsum = r;
}

// Statistics of n contiguous elements starting at p (any alignment).
template <typename T>
__device__ __forceinline__ void row_stats(const T* __restrict__ p, int64_t n, bool ls,
                                          bool keep_in_l2, MS& st, float& rsum) {
  constexpr int E = Vec16<T>::E;
  const uintptr_t addr = reinterpret_cast<uintptr_t>(p);
  int64_t head = (int64_t)(((16 - (addr & 15)) & 15) / sizeof(T));
  if ((addr % sizeof(T)) != 0) head = n;  // not even element-aligned: scalar only
  if (head > n) head = n;
  for (int64_t j = threadIdx.x; j < head; j += blockDim.x) ms_add_scalar(st, rsum, to_f<T>(p[j]), ls);
  const T* pv = p + head;
  const int64_t nvec = (n - head) / E;
  const uint64_t pol = keep_in_l2 ? l2_policy_evict_last() : l2_policy_evict_first();
  int64_t v = threadIdx.x;
  // 4 independent 16-byte loads in flight per thread
  for (; v + 3 * blockDim.x < nvec; v += 4 * blockDim.x) {
    uint4 r[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) r[u] = ld_global_hint_v4(pv + (v + u * blockDim.x) * E, pol);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float f[E];
      unpack16<T>(r[u], f);
      ms_add_vec<E>(st, rsum, f, ls);
    }
  }
  for (; v < nvec; v += blockDim.x) {
    float f[E];
    unpack16<T>(ld_global_hint_v4(pv + v * E, pol), f);
    ms_add_vec<E>(st, rsum, f, ls);
  }
  for (int64_t j = head + nvec * E + threadIdx.x; j < n; j += blockDim.x)
    ms_add_scalar(st, rsum, to_f<T>(p[j]), ls);
}

// f[i] <- scale * exp2(f[i] * log2 e - lb) - se, two lanes per instruction;
// the same roundings as the scalar form (fused multiply-adds, ex2.approx).
template <int E>
__device__ __forceinline__ void grad_vec(float* f, float lb, float scale, float se) {
  const float2 l2 = make_float2(kLog2e, kLog2e), b2 = make_float2(-lb, -lb);
  const float2 s2 = make_float2(scale, scale), c2 = make_float2(-se, -se);
#pragma unroll
  for (int i = 0; i < E; i += 2) {
    const float2 a = fma2(make_float2(f[i], f[i + 1]), l2, b2);
    const float2 ex = make_float2(fast_exp2(a.x), fast_exp2(a.y));
    const float2 g = fma2(s2, ex, c2);
    f[i] = g.x;
    f[i + 1] = g.y;
  }
}

// Writes g[j] = scale * (exp(x[j] - lse) - eps_v - (1-e)[j + col0 == t]) for j < n.
// scale == 0 (ignored row) writes zeros without reading x.
template <typename T>
__device__ __forceinline__ void row_grad(const T* __restrict__ p, T* __restrict__ g, int64_t n,
                                         int64_t col0, int64_t t, float lse, float scale,
                                         float eps_v, float one_m_e) {
  constexpr int E = Vec16<T>::E;
  const float lb = lse * kLog2e;
  const float se = scale * eps_v;
  const uintptr_t ap = reinterpret_cast<uintptr_t>(p), ag = reinterpret_cast<uintptr_t>(g);
  const bool vec = ((ap & 15) == (ag & 15)) && (ap % sizeof(T)) == 0;
  int64_t head = vec ? (int64_t)(((16 - (ap & 15)) & 15) / sizeof(T)) : n;
  if (head > n) head = n;
  // the one-hot term of the target column is added by fix_target() afterwards
  auto one = [&](int64_t j, float x) -> float {
    (void)j;
    return (scale == 0.f) ? 0.f : scale * fast_exp2(fmaf(x, kLog2e, -lb)) - se;
  };
  for (int64_t j = threadIdx.x; j < head; j += blockDim.x)
    g[j] = from_f<T>(one(j, scale == 0.f ? 0.f : to_f<T>(p[j])));
  const int64_t nvec = (n - head) / E;
  const T* pv = p + head;
  T* gv = g + head;
  const uint64_t pol = l2_policy_evict_first();
  int64_t v = threadIdx.x;
  for (; v + 3 * blockDim.x < nvec; v += 4 * blockDim.x) {
    uint4 r[4];
    if (scale != 0.f) {
#pragma unroll
      for (int u = 0; u < 4; ++u) r[u] = ld_global_hint_v4(pv + (v + u * blockDim.x) * E, pol);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float f[E];
      if (scale != 0.f) {
        unpack16<T>(r[u], f);
        grad_vec<E>(f, lb, scale, se);
      } else {
#pragma unroll
        for (int i = 0; i < E; ++i) f[i] = 0.f;
      }
      st_global_stream_v4(gv + (v + u * blockDim.x) * E, pack16<T>(f));
    }
  }
  for (; v < nvec; v += blockDim.x) {
    float f[E];
    if (scale != 0.f) unpack16<T>(ld_global_hint_v4(pv + v * E, pol), f);
    const int64_t j0 = head + v * E;
#pragma unroll
    for (int i = 0; i < E; ++i) f[i] = one(j0 + i, scale != 0.f ? f[i] : 0.f);
    st_global_stream_v4(gv + v * E, pack16<T>(f));
  }
  for (int64_t j = head + nvec * E + threadIdx.x; j < n; j += blockDim.x)
    g[j] = from_f<T>(one(j, scale == 0.f ? 0.f : to_f<T>(p[j])));
}

// Rewrites the target element of a gradient row with its one-hot term.  Called
// by every thread after row_grad; the CTA barrier orders it after the vector
// store that wrote the same element.
template <typename T>
__device__ __forceinline__ void fix_target(const T* __restrict__ p, T* __restrict__ g, int64_t n,
                                           int64_t col0, int64_t t, float lse, float scale,
                                           float eps_v, float one_m_e) {
  __syncthreads();
  const int64_t j = t - col0;
  if (threadIdx.x == 0 && scale != 0.f && j >= 0 && j < n) {
    const float x = to_f<T>(p[j]);
    const float v = scale * fast_exp2(fmaf(x, kLog2e, -lse * kLog2e)) - scale * eps_v -
                    scale * one_m_e;
    g[j] = from_f<T>(v);
  }
}

// n_valid = #(target != ignore_index), written as float.
__global__ void ce_count_valid_kernel(const int64_t* __restrict__ target, int64_t B,
                                      int64_t ignore_index, float* __restrict__ n_valid) {
  __shared__ float red[32];
  float c = 0.f;
  for (int64_t b = threadIdx.x; b < B; b += blockDim.x) c += (target[b] != ignore_index) ? 1.f : 0.f;
  c = block_sum(c, red);
  if (threadIdx.x == 0) *n_valid = c;
}

__device__ __forceinline__ float read_scalar(const void* p, int dt, int64_t i) {
  switch (dt) {
    case FO_F32: return reinterpret_cast<const float*>(p)[i];
    case FO_F16: return __half2float(reinterpret_cast<const __half*>(p)[i]);
    case FO_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    case FO_F64: return (float)reinterpret_cast<const double*>(p)[i];
  }
  return 0.f;
}

template <typename T, bool LS>
__global__ void __launch_bounds__(kThreads)
ce_fwd_kernel(const T* __restrict__ logits, const int64_t* __restrict__ target,
              float* __restrict__ loss_rows, float* __restrict__ lse_out, T* __restrict__ dlogits,
              const float* __restrict__ n_valid, int64_t B, int64_t V, int64_t ld,
              int64_t ignore_index, float eps, int reduction) {
  __shared__ float sm[96];
  __shared__ float s_lse;
  const bool grad = dlogits != nullptr;
  for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
    const T* row = logits + b * ld;
    const int64_t t = target[b];
    const bool valid = (t != ignore_index);
    MS st{-INFINITY, 0.f};
    float rsum = 0.f;
    l2_prefetch(row, V * (int64_t)sizeof(T));
    row_stats<T>(row, V, LS, grad, st, rsum);
    block_ms(st, rsum, sm);
    if (threadIdx.x == 0) {
      const float lse = st.m + logf(st.s);
      float loss = 0.f;
      if (valid) {
        const float xt = (t >= 0 && t < V) ? to_f<T>(row[t]) : NAN;
        loss = lse - (1.f - eps) * xt;
        if (LS) loss -= eps * (rsum / (float)V);
      }
      loss_rows[b] = loss;
      lse_out[b] = lse;
      s_lse = lse;
    }
    if (grad) {
      __syncthreads();
      const float lse = s_lse;
      float scale = valid ? 1.f : 0.f;
      if (valid && reduction == FO_RED_MEAN) scale = 1.f / *n_valid;
      row_grad<T>(row, dlogits + b * V, V, 0, t, lse, scale, LS ? eps / (float)V : 0.f,
                  1.f - eps);
      fix_target<T>(row, dlogits + b * V, V, 0, t, lse, scale, LS ? eps / (float)V : 0.f,
                    1.f - eps);
    }
  }
}

// Deterministic single-CTA reduction of loss_rows -> out_scalar (sum or mean).
__global__ void ce_reduce_kernel(const float* __restrict__ loss_rows, int64_t B,
                                 const float* __restrict__ n_valid, int reduction,
                                 float* __restrict__ out_scalar) {
  __shared__ float red[32];
  float s = 0.f;
  for (int64_t b = threadIdx.x; b < B; b += blockDim.x) s += loss_rows[b];
  s = block_sum(s, red);
  if (threadIdx.x == 0) *out_scalar = (reduction == FO_RED_MEAN) ? s / *n_valid : s;
}

template <typename T, bool LS>
__global__ void __launch_bounds__(kThreads)
ce_bwd_kernel(const T* __restrict__ logits, const int64_t* __restrict__ target,
              const float* __restrict__ lse, const void* __restrict__ dout, int dout_dtype,
              int dout_is_vector, const float* __restrict__ n_valid, T* __restrict__ dlogits,
              int64_t B, int64_t Vn, int64_t ld, int64_t col0, int64_t V, int64_t ignore_index,
              float eps, int reduction) {
  for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
    const int64_t t = target[b];
    const bool valid = (t != ignore_index);
    float scale = 0.f;
    if (valid) {
      scale = read_scalar(dout, dout_dtype, dout_is_vector ? b : 0);
      if (reduction == FO_RED_MEAN) scale /= *n_valid;
    }
    row_grad<T>(logits + b * ld, dlogits + b * Vn, Vn, col0, t, lse[b], scale,
                LS ? eps / (float)V : 0.f, 1.f - eps);
    fix_target<T>(logits + b * ld, dlogits + b * Vn, Vn, col0, t, lse[b], scale,
                  LS ? eps / (float)V : 0.f, 1.f - eps);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
ce_scale_kernel(T* __restrict__ g, const void* __restrict__ dout, int dout_dtype, int is_vec,
                int64_t B, int64_t V, int64_t ld) {
  if (!is_vec) {
    const float d = read_scalar(dout, dout_dtype, 0);
    if (d == 1.0f) return;  // backward of loss.backward(): nothing to scale
  }
  constexpr int E = Vec16<T>::E;
  for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
    const float d = read_scalar(dout, dout_dtype, is_vec ? b : 0);
    T* row = g + b * ld;
    const uintptr_t a = reinterpret_cast<uintptr_t>(row);
    int64_t head = (a % sizeof(T)) ? V : (int64_t)(((16 - (a & 15)) & 15) / sizeof(T));
    if (head > V) head = V;
    for (int64_t j = threadIdx.x; j < head; j += blockDim.x) row[j] = from_f<T>(to_f<T>(row[j]) * d);
    const int64_t nvec = (V - head) / E;
    T* rv = row + head;
    for (int64_t v = threadIdx.x; v < nvec; v += blockDim.x) {
      float f[E];
      unpack16<T>(ld_global_stream_v4(rv + v * E), f);
#pragma unroll
      for (int i = 0; i < E; ++i) f[i] *= d;
      st_global_stream_v4(rv + v * E, pack16<T>(f));
    }
    for (int64_t j = head + nvec * E + threadIdx.x; j < V; j += blockDim.x)
      row[j] = from_f<T>(to_f<T>(row[j]) * d);
  }
}

// Vocabulary shard: per-row (max, sumexp, target logit or 0, row sum).
template <typename T>
__global__ void __launch_bounds__(kThreads)
ce_shard_stats_kernel(const T* __restrict__ logits, const int64_t* __restrict__ target,
                      float* __restrict__ stats, int64_t B, int64_t Vn, int64_t ld, int64_t col0,
                      int64_t ignore_index) {
  __shared__ float sm[96];
  for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
    const T* row = logits + b * ld;
    MS st{-INFINITY, 0.f};
    float rsum = 0.f;
    row_stats<T>(row, Vn, true, false, st, rsum);
    block_ms(st, rsum, sm);
    if (threadIdx.x == 0) {
      const int64_t t = target[b];
      float xt = 0.f;
      if (t != ignore_index && t >= col0 && t < col0 + Vn) xt = to_f<T>(row[t - col0]);
      stats[b * 4 + 0] = st.m;
      stats[b * 4 + 1] = st.s;
      stats[b * 4 + 2] = xt;
      stats[b * 4 + 3] = rsum;
    }
  }
}

__global__ void ce_shard_combine_kernel(const float* __restrict__ all, int P,
                                        const int64_t* __restrict__ target,
                                        float* __restrict__ loss_rows, float* __restrict__ lse_out,
                                        int64_t B, int64_t V, int64_t ignore_index, float eps) {
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < B;
       b += (int64_t)gridDim.x * blockDim.x) {
    MS st{-INFINITY, 0.f};
    float xt = 0.f, rsum = 0.f;
    for (int p = 0; p < P; ++p) {
      const float* s = all + ((int64_t)p * B + b) * 4;
      st = ms_merge(st, MS{s[0], s[1]});
      xt += s[2];
      rsum += s[3];
    }
    const float lse = st.m + logf(st.s);
    const int64_t t = target[b];
    float loss = 0.f;
    if (t != ignore_index) {
      loss = (t >= 0 && t < V) ? lse - (1.f - eps) * xt : NAN;
      if (eps != 0.f) loss -= eps * (rsum / (float)V);
    }
    loss_rows[b] = loss;
    lse_out[b] = lse;
  }
}

int grid_rows(int64_t B, int per_sm) {
  int64_t g = (int64_t)num_sms() * per_sm;
  return (int)(g < B ? g : B);
}

template <typename T>
int ce_fwd_t(const void* logits, const int64_t* target, float* loss_rows, float* lse,
             float* out_scalar, float* n_valid, void* dlogits, int64_t B, int64_t V, int64_t ld,
             int64_t ignore_index, float eps, int reduction, cudaStream_t st) {
  ce_count_valid_kernel<<<1, 1024, 0, st>>>(target, B, ignore_index, n_valid);
  if (int rc = check_launch("ce_count_valid_kernel")) return rc;
  // with the gradient fused, pass 2 re-reads each row from L2: keep the rows in
  // flight (CTAs x 250 KB for V = 128K bf16) well inside the 126 MB L2
  const int grid = grid_rows(B, dlogits ? 2 : 4);
  if (eps != 0.f)
    ce_fwd_kernel<T, true><<<grid, kThreads, 0, st>>>((const T*)logits, target, loss_rows, lse,
                                                      (T*)dlogits, n_valid, B, V, ld,
                                                      ignore_index, eps, reduction);
  else
    ce_fwd_kernel<T, false><<<grid, kThreads, 0, st>>>((const T*)logits, target, loss_rows, lse,
                                                       (T*)dlogits, n_valid, B, V, ld,
                                                       ignore_index, eps, reduction);
  if (int rc = check_launch("ce_fwd_kernel")) return rc;
  if (reduction != FO_RED_NONE) {
    ce_reduce_kernel<<<1, 1024, 0, st>>>(loss_rows, B, n_valid, reduction, out_scalar);
    return check_launch("ce_reduce_kernel");
  }
  return FO_OK;
}

template <typename T>
int ce_bwd_t(const void* logits, const int64_t* target, const float* lse, const void* dout,
             int dout_dtype, int dout_is_vector, const float* n_valid, void* dlogits, int64_t B,
             int64_t Vn, int64_t ld, int64_t col0, int64_t V, int64_t ignore_index, float eps,
             int reduction, cudaStream_t st) {
  const int grid = grid_rows(B, 4);
  if (eps != 0.f)
    ce_bwd_kernel<T, true><<<grid, kThreads, 0, st>>>(
        (const T*)logits, target, lse, dout, dout_dtype, dout_is_vector, n_valid, (T*)dlogits, B,
        Vn, ld, col0, V, ignore_index, eps, reduction);
  else
    ce_bwd_kernel<T, false><<<grid, kThreads, 0, st>>>(
        (const T*)logits, target, lse, dout, dout_dtype, dout_is_vector, n_valid, (T*)dlogits, B,
        Vn, ld, col0, V, ignore_index, eps, reduction);
  return check_launch("ce_bwd_kernel");
}


// ---------------------------------------------------------------------------
// Vocabulary-sharded forward (+ gradient) as one kernel over NVLink peer memory
// ---------------------------------------------------------------------------
// Each rank owns a region of the same layout, mapped into every other rank's
// address space (CUDA IPC); capacity Bc rows:
//   stats [2][P][Bc] float4   (max, sum exp(x - max), target logit or 0, row sum)
//                              of source rank p for row b, double-buffered by
//                              the call's epoch parity
//   flags [P][Bc] uint32       epoch of the call whose stats of (p, b) landed
// A CTA computes the statistics of its row (the row stays in L2: evict_last),
// stores them into every rank's region (P2P stores) and publishes each with a
// system-scope release store of the epoch into that rank's flag.  `lag` rows
// later (0 or 1) it acquires the P flags of that row in its own region,
// combines the statistics in rank order (the same result on every rank) and
// writes that row's gradient slice, re-reading the row from L2.  Forward +
// gradient cost one HBM read and one write of the rank's [B, V_local] block.
// With lag 1 the exchange (16 bytes per row and rank) overlaps the next row's
// statistics, at the price of two rows per CTA held in L2; the host picks lag 1
// when that fits (short rows, many ranks), else lag 0, where the other CTAs of
// the SM cover the wait.
// Ranks run the same persistent grid over the same rows, so a CTA waits only on
// rows its counterparts on the other GPUs process at the same time.  Waits are
// bounded: one that runs out counts in g_ce_p2p_timeouts, marks the epoch as
// failed (every later wait of the call gives up at once) and leaves that row's
// loss NaN.  Parity double-buffering keeps a rank that starts call k + 1 from
// overwriting statistics a slower rank still reads in call k (a rank cannot get
// two calls ahead: call k + 1 needs every rank's call-(k + 1) statistics).
__device__ unsigned int g_ce_p2p_timeouts;
__device__ unsigned int g_ce_p2p_failed_epoch;
constexpr uint32_t kP2PWaitLimit = 1u << 22;
constexpr int kP2PMaxRanks = 8;

struct PeerRegions {
  void* r[kP2PMaxRanks];
};

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr int kP2PThreads = 256;  // 4 CTAs per SM: the shard rows are short

template <typename T, bool LS>
__global__ void __launch_bounds__(kP2PThreads)
ce_shard_p2p_kernel(const T* __restrict__ logits, const int64_t* __restrict__ target,
                    float* __restrict__ loss_rows, float* __restrict__ lse_out,
                    T* __restrict__ dlogits, const float* __restrict__ n_valid, int64_t B,
                    int64_t Vn, int64_t ld, int64_t col0, int64_t V, int64_t ignore_index,
                    float eps, int reduction, PeerRegions peers, int P, int rank, int64_t Bc,
                    uint32_t epoch, int lag) {
  __shared__ float sm[96];
  __shared__ float4 s_st[kP2PMaxRanks];
  __shared__ int s_bad;
  const bool grad = dlogits != nullptr;
  const int par = (int)(epoch & 1u);
  const int64_t G = gridDim.x;
  const int64_t nmine = B > (int64_t)blockIdx.x ? (B - 1 - blockIdx.x) / G + 1 : 0;
  float4* own_stats = reinterpret_cast<float4*>(peers.r[rank]);
  const uint32_t* own_flags =
      reinterpret_cast<const uint32_t*>(own_stats + 2 * (int64_t)P * Bc);
  for (int64_t j = 0; j < nmine + lag; ++j) {
    if (j < nmine) {
      // ---- statistics of row j, published to every rank
      const int64_t b = blockIdx.x + j * G;
      const T* row = logits + b * ld;
      MS st{-INFINITY, 0.f};
      float rsum = 0.f;
      l2_prefetch(row, Vn * (int64_t)sizeof(T));
      row_stats<T>(row, Vn, LS, grad, st, rsum);
      block_ms(st, rsum, sm);
      if (threadIdx.x < P) {
        const int q = threadIdx.x;
        const int64_t t = target[b];
        float xt = 0.f;
        if (t != ignore_index && t >= col0 && t < col0 + Vn) xt = to_f<T>(row[t - col0]);
        float4* qs = reinterpret_cast<float4*>(peers.r[q]);
        uint32_t* qf = reinterpret_cast<uint32_t*>(qs + 2 * (int64_t)P * Bc);
        qs[((int64_t)par * P + rank) * Bc + b] = make_float4(st.m, st.s, xt, rsum);
        st_release_sys_u32(qf + (int64_t)rank * Bc + b, epoch);
      }
    }
    if (j >= lag) {
      // ---- row j - lag: every rank's statistics, combine, gradient slice
      const int64_t b = blockIdx.x + (j - lag) * G;
      if (threadIdx.x == 0) s_bad = 0;
      __syncthreads();
      if (threadIdx.x < P) {
        const int p = threadIdx.x;
        const uint32_t* f = own_flags + (int64_t)p * Bc + b;
        bool ok = true;
        for (uint32_t n = 0; ld_acquire_sys_u32(f) != epoch; ++n) {
          if (n >= kP2PWaitLimit || *reinterpret_cast<volatile uint32_t*>(&g_ce_p2p_failed_epoch) ==
                                        epoch) {
            ok = false;
            break;
          }
        }
        if (ok) {
          s_st[p] = __ldcg(own_stats + ((int64_t)par * P + p) * Bc + b);
        } else {
          if (atomicExch(&g_ce_p2p_failed_epoch, epoch) != epoch) atomicAdd(&g_ce_p2p_timeouts, 1u);
          s_bad = 1;
        }
      }
      __syncthreads();
      MS st{-INFINITY, 0.f};
      float xt = 0.f, rsum = 0.f;
      for (int p = 0; p < P; ++p) {
        const float4 v = s_st[p];
        st = ms_merge(st, MS{v.x, v.y});
        xt += v.z;
        rsum += v.w;
      }
      const float lse = s_bad ? NAN : st.m + logf(st.s);
      const int64_t t = target[b];
      const bool valid = (t != ignore_index);
      if (threadIdx.x == 0) {
        float loss = 0.f;
        if (valid) {
          loss = (t >= 0 && t < V) ? lse - (1.f - eps) * xt : NAN;
          if (LS) loss -= eps * (rsum / (float)V);
        }
        loss_rows[b] = s_bad ? NAN : loss;
        lse_out[b] = lse;
      }
      if (grad) {
        float scale = valid ? 1.f : 0.f;
        if (valid && reduction == FO_RED_MEAN) scale = 1.f / *n_valid;
        const T* row = logits + b * ld;
        row_grad<T>(row, dlogits + b * Vn, Vn, col0, t, lse, scale, LS ? eps / (float)V : 0.f,
                    1.f - eps);
        fix_target<T>(row, dlogits + b * Vn, Vn, col0, t, lse, scale, LS ? eps / (float)V : 0.f,
                      1.f - eps);
      }
      __syncthreads();  // s_st / s_bad are rewritten for the next row
    }
  }
}


// Short shard rows (<= 32 KiB: the vocabulary split over 8 or more ranks): one
// warp per row instead of one CTA, so a row's reductions are warp shuffles and
// an SM keeps 16-32 rows in flight (the whole row is requested from L2 by bulk
// prefetches, which supplies the memory parallelism).  Same exchange as
// ce_shard_p2p_kernel with lag 0: the warp publishes its row's statistics,
// waits for the other ranks' of the same row (the other warps of the SM cover
// the wait) and writes the gradient slice from L2.
template <typename T>
__device__ __forceinline__ void warp_row_stats(const T* __restrict__ p, int64_t n, bool ls,
                                               uint64_t pol, int lane, MS& st, float& rsum) {
  constexpr int E = Vec16<T>::E;
  const uintptr_t addr = reinterpret_cast<uintptr_t>(p);
  int64_t head = (int64_t)(((16 - (addr & 15)) & 15) / sizeof(T));
  if ((addr % sizeof(T)) != 0) head = n;
  if (head > n) head = n;
  for (int64_t j = lane; j < head; j += 32) ms_add_scalar(st, rsum, to_f<T>(p[j]), ls);
  const T* pv = p + head;
  const int64_t nvec = (n - head) / E;
  int64_t v = lane;
  for (; v + 96 < nvec; v += 128) {
    uint4 r[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) r[u] = ld_global_hint_v4(pv + (v + 32 * u) * E, pol);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float f[E];
      unpack16<T>(r[u], f);
      ms_add_vec<E>(st, rsum, f, ls);
    }
  }
  for (; v < nvec; v += 32) {
    float f[E];
    unpack16<T>(ld_global_hint_v4(pv + v * E, pol), f);
    ms_add_vec<E>(st, rsum, f, ls);
  }
  for (int64_t j = head + nvec * E + lane; j < n; j += 32) ms_add_scalar(st, rsum, to_f<T>(p[j]), ls);
}

template <typename T>
__device__ __forceinline__ void warp_row_grad(const T* __restrict__ p, T* __restrict__ g, int64_t n,
                                              float lse, float scale, float eps_v, int lane) {
  constexpr int E = Vec16<T>::E;
  const float lb = lse * kLog2e;
  const float se = scale * eps_v;
  const uintptr_t ap = reinterpret_cast<uintptr_t>(p), ag = reinterpret_cast<uintptr_t>(g);
  const bool vec = ((ap & 15) == (ag & 15)) && (ap % sizeof(T)) == 0;
  int64_t head = vec ? (int64_t)(((16 - (ap & 15)) & 15) / sizeof(T)) : n;
  if (head > n) head = n;
  auto one = [&](float x) -> float {
    return (scale == 0.f) ? 0.f : scale * fast_exp2(fmaf(x, kLog2e, -lb)) - se;
  };
  for (int64_t j = lane; j < head; j += 32)
    g[j] = from_f<T>(one(scale == 0.f ? 0.f : to_f<T>(p[j])));
  const int64_t nvec = (n - head) / E;
  const T* pv = p + head;
  T* gv = g + head;
  const uint64_t pol = l2_policy_evict_first();
  int64_t v = lane;
  for (; v + 96 < nvec; v += 128) {
    uint4 r[4];
    if (scale != 0.f) {
#pragma unroll
      for (int u = 0; u < 4; ++u) r[u] = ld_global_hint_v4(pv + (v + 32 * u) * E, pol);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float f[E];
      if (scale != 0.f) {
        unpack16<T>(r[u], f);
        grad_vec<E>(f, lb, scale, se);
      } else {
#pragma unroll
        for (int i = 0; i < E; ++i) f[i] = 0.f;
      }
      st_global_stream_v4(gv + (v + 32 * u) * E, pack16<T>(f));
    }
  }
  for (; v < nvec; v += 32) {
    float f[E];
    if (scale != 0.f) unpack16<T>(ld_global_hint_v4(pv + v * E, pol), f);
#pragma unroll
    for (int i = 0; i < E; ++i) f[i] = one(scale != 0.f ? f[i] : 0.f);
    st_global_stream_v4(gv + v * E, pack16<T>(f));
  }
  for (int64_t j = head + nvec * E + lane; j < n; j += 32)
    g[j] = from_f<T>(one(scale == 0.f ? 0.f : to_f<T>(p[j])));
}

constexpr int kP2PWarps = 8;

template <typename T, bool LS>
__global__ void __launch_bounds__(32 * kP2PWarps)
ce_shard_p2p_warp_kernel(const T* __restrict__ logits, const int64_t* __restrict__ target,
                         float* __restrict__ loss_rows, float* __restrict__ lse_out,
                         T* __restrict__ dlogits, const float* __restrict__ n_valid, int64_t B,
                         int64_t Vn, int64_t ld, int64_t col0, int64_t V, int64_t ignore_index,
                         float eps, int reduction, PeerRegions peers, int P, int rank, int64_t Bc,
                         uint32_t epoch) {
  const int lane = threadIdx.x & 31;
  const bool grad = dlogits != nullptr;
  const int par = (int)(epoch & 1u);
  const int64_t W = (int64_t)gridDim.x * kP2PWarps;
  float4* own_stats = reinterpret_cast<float4*>(peers.r[rank]);
  const uint32_t* own_flags =
      reinterpret_cast<const uint32_t*>(own_stats + 2 * (int64_t)P * Bc);
  const uint64_t pol = grad ? l2_policy_evict_last() : l2_policy_evict_first();
  const float scale_mean = (reduction == FO_RED_MEAN && grad) ? 1.f / *n_valid : 1.f;
  for (int64_t b = (int64_t)blockIdx.x * kP2PWarps + (threadIdx.x >> 5); b < B; b += W) {
    const T* row = logits + b * ld;
    {
      // the whole row requested from L2 at once, pieces of at most 32 KiB
      const uintptr_t a = reinterpret_cast<uintptr_t>(row);
      const uintptr_t a0 = (a + 15) & ~(uintptr_t)15;
      const uintptr_t a1 = (a + (uintptr_t)(Vn * (int64_t)sizeof(T))) & ~(uintptr_t)15;
      for (uintptr_t off = (uintptr_t)lane * 32768; a0 + off < a1; off += 32 * 32768) {
        const uintptr_t nb = (a1 - a0 - off) < 32768 ? (a1 - a0 - off) : 32768;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a0 + off),
                     "r"((uint32_t)nb)
                     : "memory");
      }
    }
    MS st{-INFINITY, 0.f};
    float rsum = 0.f;
    warp_row_stats<T>(row, Vn, LS, pol, lane, st, rsum);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      MS other{__shfl_xor_sync(0xffffffffu, st.m, o), __shfl_xor_sync(0xffffffffu, st.s, o)};
      st = ms_merge(st, other);
      if (LS) rsum += __shfl_xor_sync(0xffffffffu, rsum, o);
    }
    const int64_t t = target[b];
    const bool valid = (t != ignore_index);
    if (lane < P) {
      float xt = 0.f;
      if (valid && t >= col0 && t < col0 + Vn) xt = to_f<T>(row[t - col0]);
      float4* qs = reinterpret_cast<float4*>(peers.r[lane]);
      uint32_t* qf = reinterpret_cast<uint32_t*>(qs + 2 * (int64_t)P * Bc);
      qs[((int64_t)par * P + rank) * Bc + b] = make_float4(st.m, st.s, xt, rsum);
      st_release_sys_u32(qf + (int64_t)rank * Bc + b, epoch);
    }
    // every rank's statistics of row b (lane p polls rank p's flag)
    float4 mine = make_float4(-INFINITY, 0.f, 0.f, 0.f);
    int bad = 0;
    if (lane < P) {
      const uint32_t* f = own_flags + (int64_t)lane * Bc + b;
      bool ok = true;
      for (uint32_t n = 0; ld_acquire_sys_u32(f) != epoch; ++n) {
        if (n >= kP2PWaitLimit ||
            *reinterpret_cast<volatile uint32_t*>(&g_ce_p2p_failed_epoch) == epoch) {
          ok = false;
          break;
        }
      }
      if (ok) {
        mine = __ldcg(own_stats + ((int64_t)par * P + lane) * Bc + b);
      } else {
        if (atomicExch(&g_ce_p2p_failed_epoch, epoch) != epoch) atomicAdd(&g_ce_p2p_timeouts, 1u);
        bad = 1;
      }
    }
    bad = __any_sync(0xffffffffu, bad);
    MS c{-INFINITY, 0.f};
    float xt = 0.f, rs = 0.f;
    for (int p = 0; p < P; ++p) {  // rank order: the same result on every rank
      c = ms_merge(c, MS{__shfl_sync(0xffffffffu, mine.x, p), __shfl_sync(0xffffffffu, mine.y, p)});
      xt += __shfl_sync(0xffffffffu, mine.z, p);
      rs += __shfl_sync(0xffffffffu, mine.w, p);
    }
    const float lse = bad ? NAN : c.m + logf(c.s);
    if (lane == 0) {
      float loss = 0.f;
      if (valid) {
        loss = (t >= 0 && t < V) ? lse - (1.f - eps) * xt : NAN;
        if (LS) loss -= eps * (rs / (float)V);
      }
      loss_rows[b] = bad ? NAN : loss;
      lse_out[b] = lse;
    }
    if (grad) {
      const float scale = valid ? scale_mean : 0.f;
      const float eps_v = LS ? eps / (float)V : 0.f;
      T* grow = dlogits + b * Vn;
      warp_row_grad<T>(row, grow, Vn, lse, scale, eps_v, lane);
      __syncwarp();  // the vector store of the target element lands before its fix
      const int64_t j = t - col0;
      if (lane == 0 && scale != 0.f && j >= 0 && j < Vn) {
        const float x = to_f<T>(row[j]);
        grow[j] = from_f<T>(scale * fast_exp2(fmaf(x, kLog2e, -lse * kLog2e)) - scale * eps_v -
                            scale * (1.f - eps));
      }
    }
  }
}

template <typename T>
int ce_shard_p2p_t(const void* logits, const int64_t* target, float* loss_rows, float* lse,
                   float* out_scalar, float* n_valid, void* dlogits, int64_t B, int64_t Vn,
                   int64_t ld, int64_t col0, int64_t V, int64_t ignore_index, float eps,
                   int reduction, const PeerRegions& peers, int P, int rank, int64_t Bc,
                   uint32_t epoch, cudaStream_t st) {
  ce_count_valid_kernel<<<1, 1024, 0, st>>>(target, B, ignore_index, n_valid);
  if (int rc = check_launch("ce_count_valid_kernel")) return rc;
  const double row_bytes = (double)Vn * sizeof(T);
  if (row_bytes <= 32768.0) {
    // short rows: a warp per row, up to ~120 MB of rows between their two reads
    // (measured at 32 KiB rows on two B200s: 2 CTAs per SM 0.221 ms, 3 CTAs
    // 0.211 ms; the all-gather path 0.296 ms; at 64 KiB rows the CTA-per-row
    // kernel below, 0.364 ms, beat the warp kernel's 0.502 ms)
    auto wk = eps != 0.f ? ce_shard_p2p_warp_kernel<T, true> : ce_shard_p2p_warp_kernel<T, false>;
    int occ = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, wk, 32 * kP2PWarps, 0);
    int per_sm = (int)(120.0 * (1 << 20) / (row_bytes * kP2PWarps * num_sms()));
    if (per_sm > occ) per_sm = occ;
    if (per_sm > 4) per_sm = 4;
    if (per_sm < 1) per_sm = 1;
    const int64_t need = (B + kP2PWarps - 1) / kP2PWarps;
    int64_t grid = (int64_t)num_sms() * per_sm;
    if (grid > need) grid = need;
    wk<<<(unsigned)grid, 32 * kP2PWarps, 0, st>>>((const T*)logits, target, loss_rows, lse,
                                                  (T*)dlogits, n_valid, B, Vn, ld, col0, V,
                                                  ignore_index, eps, reduction, peers, P, rank, Bc,
                                                  epoch);
    if (int rc = check_launch("ce_shard_p2p_warp_kernel")) return rc;
    if (reduction != FO_RED_NONE) {
      ce_reduce_kernel<<<1, 1024, 0, st>>>(loss_rows, B, n_valid, reduction, out_scalar);
      return check_launch("ce_reduce_kernel");
    }
    return FO_OK;
  }
  // every CTA resident at once (a CTA waits only on its counterparts on other
  // GPUs, which run the same grid); rows held in L2 (grid x (1 + lag) rows,
  // evict_last) kept under ~72 MB of the 126 MB
  auto kern = eps != 0.f ? ce_shard_p2p_kernel<T, true> : ce_shard_p2p_kernel<T, false>;
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kP2PThreads, 0);
  if (per_sm < 1) per_sm = 1;
  if (per_sm > 4) per_sm = 4;
  const int grid = grid_rows(B, per_sm);
  const int lag = (dlogits && (double)grid * 2.0 * row_bytes <= 72.0 * (1 << 20)) ? 1 : 0;
  kern<<<grid, kP2PThreads, 0, st>>>((const T*)logits, target, loss_rows, lse, (T*)dlogits,
                                     n_valid, B, Vn, ld, col0, V, ignore_index, eps, reduction,
                                     peers, P, rank, Bc, epoch, lag);
  if (int rc = check_launch("ce_shard_p2p_kernel")) return rc;
  if (reduction != FO_RED_NONE) {
    ce_reduce_kernel<<<1, 1024, 0, st>>>(loss_rows, B, n_valid, reduction, out_scalar);
    return check_launch("ce_reduce_kernel");
  }
  return FO_OK;
}

int check_common(const void* logits, const void* target, int64_t B, int64_t V, int64_t ld,
                 int dtype, const char* op) {
  FO_CHECK_ARG(B >= 0 && V > 0 && ld >= V, "%s: bad shape B=%lld V=%lld ld=%lld", op,
               (long long)B, (long long)V, (long long)ld);
  FO_CHECK_ARG(B == 0 || (logits && target), "%s: null pointer", op);
  if (dtype != FO_F32 && dtype != FO_F16 && dtype != FO_BF16) {
    set_error("%s: unsupported logits dtype code %d", op, dtype);
    return FO_EDTYPE;
  }
  return FO_OK;
}

}  // namespace
}  // namespace fo

using namespace fo;

extern "C" int fo_ce_workspace_bytes(int64_t B, int64_t* bytes) {
  clear_error();
  FO_CHECK_ARG(bytes && B >= 0, "fo_ce_workspace_bytes: bad argument");
  *bytes = 0;
  return FO_OK;
}

extern "C" int fo_ce_fwd(const void* logits, const int64_t* target, float* loss_rows, float* lse,
                         float* out_scalar, float* n_valid_out, void* dlogits, int64_t B,
                         int64_t V, int64_t ld, int64_t ignore_index, float label_smoothing,
                         int reduction, int dtype, void* workspace, int64_t ws_bytes,
                         void* stream) {
  (void)workspace;
  (void)ws_bytes;
  clear_error();
  if (int rc = check_common(logits, target, B, V, ld, dtype, "fo_ce_fwd")) return rc;
  FO_CHECK_ARG(reduction >= FO_RED_NONE && reduction <= FO_RED_SUM, "fo_ce_fwd: bad reduction %d",
               reduction);
  FO_CHECK_ARG(n_valid_out && (B == 0 || (loss_rows && lse)), "fo_ce_fwd: null output pointer");
  FO_CHECK_ARG(reduction == FO_RED_NONE || out_scalar, "fo_ce_fwd: null out_scalar");
  FO_CHECK_ARG(label_smoothing >= 0.f && label_smoothing <= 1.f, "fo_ce_fwd: bad label_smoothing");
  cudaStream_t st = as_stream(stream);
  if (B == 0) {
    cudaMemsetAsync(n_valid_out, 0, sizeof(float), st);
    if (reduction != FO_RED_NONE) {
      ce_reduce_kernel<<<1, 32, 0, st>>>(loss_rows, 0, n_valid_out, reduction, out_scalar);
      return check_launch("ce_reduce_kernel");
    }
    return FO_OK;
  }
  switch (dtype) {
    case FO_F32:
      return ce_fwd_t<float>(logits, target, loss_rows, lse, out_scalar, n_valid_out, dlogits, B,
                             V, ld, ignore_index, label_smoothing, reduction, st);
    case FO_F16:
      return ce_fwd_t<__half>(logits, target, loss_rows, lse, out_scalar, n_valid_out, dlogits,
                              B, V, ld, ignore_index, label_smoothing, reduction, st);
    default:
      return ce_fwd_t<__nv_bfloat16>(logits, target, loss_rows, lse, out_scalar, n_valid_out,
                                     dlogits, B, V, ld, ignore_index, label_smoothing, reduction,
                                     st);
  }
}

extern "C" int fo_ce_bwd(const void* logits, const int64_t* target, const float* lse,
                         const void* dout, int dout_dtype, int dout_is_vector,
                         const float* n_valid, void* dlogits, int64_t B, int64_t V, int64_t ld,
                         int64_t ignore_index, float label_smoothing, int reduction, int dtype,
                         void* stream) {
  clear_error();
  if (int rc = check_common(logits, target, B, V, ld, dtype, "fo_ce_bwd")) return rc;
  if (B == 0) return FO_OK;
  FO_CHECK_ARG(lse && dout && dlogits && (reduction != FO_RED_MEAN || n_valid),
               "fo_ce_bwd: null pointer");
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case FO_F32:
      return ce_bwd_t<float>(logits, target, lse, dout, dout_dtype, dout_is_vector, n_valid,
                             dlogits, B, V, ld, 0, V, ignore_index, label_smoothing, reduction, st);
    case FO_F16:
      return ce_bwd_t<__half>(logits, target, lse, dout, dout_dtype, dout_is_vector, n_valid,
                              dlogits, B, V, ld, 0, V, ignore_index, label_smoothing, reduction,
                              st);
    default:
      return ce_bwd_t<__nv_bfloat16>(logits, target, lse, dout, dout_dtype, dout_is_vector,
                                     n_valid, dlogits, B, V, ld, 0, V, ignore_index,
                                     label_smoothing, reduction, st);
  }
}

extern "C" int fo_ce_scale_grad(void* dlogits, const void* dout, int dout_dtype,
                                int dout_is_vector, int64_t B, int64_t V, int64_t ld, int dtype,
                                void* stream) {
  clear_error();
  FO_CHECK_ARG(B >= 0 && V > 0 && ld >= V, "fo_ce_scale_grad: bad shape");
  if (B == 0) return FO_OK;
  FO_CHECK_ARG(dlogits && dout, "fo_ce_scale_grad: null pointer");
  cudaStream_t st = as_stream(stream);
  const int grid = grid_rows(B, 4);
  switch (dtype) {
    case FO_F32:
      ce_scale_kernel<float><<<grid, kThreads, 0, st>>>((float*)dlogits, dout, dout_dtype,
                                                        dout_is_vector, B, V, ld);
      break;
    case FO_F16:
      ce_scale_kernel<__half><<<grid, kThreads, 0, st>>>((__half*)dlogits, dout, dout_dtype,
                                                         dout_is_vector, B, V, ld);
      break;
    case FO_BF16:
      ce_scale_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(
          (__nv_bfloat16*)dlogits, dout, dout_dtype, dout_is_vector, B, V, ld);
      break;
    default:
      set_error("fo_ce_scale_grad: unsupported dtype %d", dtype);
      return FO_EDTYPE;
  }
  return check_launch("ce_scale_kernel");
}

extern "C" int fo_ce_shard_stats(const void* logits, const int64_t* target, float* stats,
                                 int64_t B, int64_t V_local, int64_t ld, int64_t v_offset,
                                 int64_t ignore_index, int dtype, void* stream) {
  clear_error();
  if (int rc = check_common(logits, target, B, V_local, ld, dtype, "fo_ce_shard_stats")) return rc;
  if (B == 0) return FO_OK;
  FO_CHECK_ARG(stats, "fo_ce_shard_stats: null stats");
  cudaStream_t st = as_stream(stream);
  const int grid = grid_rows(B, 4);
  switch (dtype) {
    case FO_F32:
      ce_shard_stats_kernel<float><<<grid, kThreads, 0, st>>>((const float*)logits, target, stats,
                                                              B, V_local, ld, v_offset,
                                                              ignore_index);
      break;
    case FO_F16:
      ce_shard_stats_kernel<__half><<<grid, kThreads, 0, st>>>(
          (const __half*)logits, target, stats, B, V_local, ld, v_offset, ignore_index);
      break;
    default:
      ce_shard_stats_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(
          (const __nv_bfloat16*)logits, target, stats, B, V_local, ld, v_offset, ignore_index);
  }
  return check_launch("ce_shard_stats_kernel");
}

extern "C" int fo_ce_shard_combine(const float* all_stats, int P, const int64_t* target,
                                   float* loss_rows, float* lse, float* out_scalar,
                                   float* n_valid_out, int64_t B, int64_t V, int64_t ignore_index,
                                   float label_smoothing, int reduction, void* stream) {
  clear_error();
  FO_CHECK_ARG(P >= 1 && B >= 0 && V > 0, "fo_ce_shard_combine: bad argument");
  FO_CHECK_ARG(loss_rows && lse && n_valid_out, "fo_ce_shard_combine: null pointer");
  cudaStream_t st = as_stream(stream);
  ce_count_valid_kernel<<<1, 1024, 0, st>>>(target, B, ignore_index, n_valid_out);
  if (int rc = check_launch("ce_count_valid_kernel")) return rc;
  if (B > 0) {
    const int grid = (int)((B + 255) / 256);
    ce_shard_combine_kernel<<<grid, 256, 0, st>>>(all_stats, P, target, loss_rows, lse, B, V,
                                                  ignore_index, label_smoothing);
    if (int rc = check_launch("ce_shard_combine_kernel")) return rc;
  }
  if (reduction != FO_RED_NONE) {
    FO_CHECK_ARG(out_scalar, "fo_ce_shard_combine: null out_scalar");
    ce_reduce_kernel<<<1, 1024, 0, st>>>(loss_rows, B, n_valid_out, reduction, out_scalar);
    return check_launch("ce_reduce_kernel");
  }
  return FO_OK;
}

extern "C" int fo_ce_shard_bwd(const void* logits, const int64_t* target, const float* lse,
                               const void* dout, int dout_dtype, int dout_is_vector,
                               const float* n_valid, void* dlogits, int64_t B, int64_t V_local,
                               int64_t ld, int64_t v_offset, int64_t V, int64_t ignore_index,
                               float label_smoothing, int reduction, int dtype, void* stream) {
  clear_error();
  if (int rc = check_common(logits, target, B, V_local, ld, dtype, "fo_ce_shard_bwd")) return rc;
  if (B == 0) return FO_OK;
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case FO_F32:
      return ce_bwd_t<float>(logits, target, lse, dout, dout_dtype, dout_is_vector, n_valid,
                             dlogits, B, V_local, ld, v_offset, V, ignore_index, label_smoothing,
                             reduction, st);
    case FO_F16:
      return ce_bwd_t<__half>(logits, target, lse, dout, dout_dtype, dout_is_vector, n_valid,
                              dlogits, B, V_local, ld, v_offset, V, ignore_index, label_smoothing,
                              reduction, st);
    default:
      return ce_bwd_t<__nv_bfloat16>(logits, target, lse, dout, dout_dtype, dout_is_vector,
                                     n_valid, dlogits, B, V_local, ld, v_offset, V, ignore_index,
                                     label_smoothing, reduction, st);
  }
}

// Row-sharded cross-entropy: this rank holds rows of the batch; n_valid_global
// (device fp32, the number of non-ignored rows over every rank, already summed
// by the caller) scales the fused gradient for 'mean'.  local_sum_out (device
// fp32, nullable for 'none') receives the sum of this rank's row losses; the
// caller sums it over ranks and divides by n_valid_global for 'mean'.
extern "C" int fo_ce_rows_fwd(const void* logits, const int64_t* target, float* loss_rows,
                              float* lse, float* local_sum_out, const float* n_valid_global,
                              void* dlogits, int64_t B, int64_t V, int64_t ld,
                              int64_t ignore_index, float label_smoothing, int reduction,
                              int dtype, void* stream) {
  clear_error();
  if (int rc = check_common(logits, target, B, V, ld, dtype, "fo_ce_rows_fwd")) return rc;
  FO_CHECK_ARG(reduction >= FO_RED_NONE && reduction <= FO_RED_SUM,
               "fo_ce_rows_fwd: bad reduction %d", reduction);
  FO_CHECK_ARG(n_valid_global && (B == 0 || (loss_rows && lse)),
               "fo_ce_rows_fwd: null pointer");
  FO_CHECK_ARG(reduction == FO_RED_NONE || local_sum_out, "fo_ce_rows_fwd: null local_sum_out");
  FO_CHECK_ARG(label_smoothing >= 0.f && label_smoothing <= 1.f,
               "fo_ce_rows_fwd: bad label_smoothing");
  cudaStream_t st = as_stream(stream);
  if (B > 0) {
    const int grid = grid_rows(B, dlogits ? 2 : 4);
#define FO_ROWS_FWD(T)                                                                         \
  if (label_smoothing != 0.f)                                                                  \
    ce_fwd_kernel<T, true><<<grid, kThreads, 0, st>>>((const T*)logits, target, loss_rows, lse, \
                                                      (T*)dlogits, n_valid_global, B, V, ld,   \
                                                      ignore_index, label_smoothing, reduction); \
  else                                                                                         \
    ce_fwd_kernel<T, false><<<grid, kThreads, 0, st>>>((const T*)logits, target, loss_rows,    \
                                                       lse, (T*)dlogits, n_valid_global, B, V, \
                                                       ld, ignore_index, label_smoothing,      \
                                                       reduction)
    switch (dtype) {
      case FO_F32: FO_ROWS_FWD(float); break;
      case FO_F16: FO_ROWS_FWD(__half); break;
      default: FO_ROWS_FWD(__nv_bfloat16); break;
    }
#undef FO_ROWS_FWD
    if (int rc = check_launch("ce_fwd_kernel")) return rc;
  }
  if (reduction != FO_RED_NONE) {
    ce_reduce_kernel<<<1, 1024, 0, st>>>(loss_rows, B, n_valid_global, FO_RED_SUM, local_sum_out);
    return check_launch("ce_reduce_kernel");
  }
  return FO_OK;
}

// n_valid_out[0] (device fp32) = number of target entries != ignore_index.
extern "C" int fo_ce_count_valid(const int64_t* target, int64_t B, int64_t ignore_index,
                                 float* n_valid_out, void* stream) {
  clear_error();
  FO_CHECK_ARG(B >= 0 && n_valid_out && (B == 0 || target), "fo_ce_count_valid: bad argument");
  ce_count_valid_kernel<<<1, 1024, 0, as_stream(stream)>>>(target, B, ignore_index, n_valid_out);
  return check_launch("ce_count_valid_kernel");
}

extern "C" int fo_ce_shard_p2p_region_bytes(int P, int64_t rows, int64_t* bytes) {
  clear_error();
  FO_CHECK_ARG(bytes && P >= 1 && P <= kP2PMaxRanks && rows >= 0,
               "fo_ce_shard_p2p_region_bytes: bad argument (1 <= P <= %d)", kP2PMaxRanks);
  *bytes = 2 * (int64_t)P * rows * 16 + (int64_t)P * rows * 4;
  return FO_OK;
}

extern "C" int fo_ce_shard_p2p_fwd(const void* logits, const int64_t* target, float* loss_rows,
                                   float* lse, float* out_scalar, float* n_valid_out,
                                   void* dlogits, int64_t B, int64_t V_local, int64_t ld,
                                   int64_t v_offset, int64_t V, int64_t ignore_index,
                                   float label_smoothing, int reduction, int dtype,
                                   void* const* regions, int P, int rank, int64_t rows_cap,
                                   uint32_t epoch, void* stream) {
  clear_error();
  if (int rc = check_common(logits, target, B, V_local, ld, dtype, "fo_ce_shard_p2p_fwd"))
    return rc;
  FO_CHECK_ARG(P >= 2 && P <= kP2PMaxRanks && rank >= 0 && rank < P && regions,
               "fo_ce_shard_p2p_fwd: bad rank layout (P=%d rank=%d)", P, rank);
  FO_CHECK_ARG(B <= rows_cap, "fo_ce_shard_p2p_fwd: %lld rows exceed the regions' %lld",
               (long long)B, (long long)rows_cap);
  FO_CHECK_ARG(epoch != 0u, "fo_ce_shard_p2p_fwd: epoch 0 is the regions' initial state");
  FO_CHECK_ARG(v_offset >= 0 && v_offset + V_local <= V, "fo_ce_shard_p2p_fwd: bad v_offset");
  FO_CHECK_ARG(loss_rows && lse && n_valid_out && (reduction == FO_RED_NONE || out_scalar),
               "fo_ce_shard_p2p_fwd: null pointer");
  PeerRegions peers{};
  for (int p = 0; p < P; ++p) {
    FO_CHECK_ARG(regions[p], "fo_ce_shard_p2p_fwd: null region of rank %d", p);
    FO_CHECK_ARG((reinterpret_cast<uintptr_t>(regions[p]) & 15) == 0,
                 "fo_ce_shard_p2p_fwd: region of rank %d not 16-byte aligned", p);
    peers.r[p] = regions[p];
  }
  if (B == 0) return FO_OK;
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case FO_F32:
      return ce_shard_p2p_t<float>(logits, target, loss_rows, lse, out_scalar, n_valid_out,
                                   dlogits, B, V_local, ld, v_offset, V, ignore_index,
                                   label_smoothing, reduction, peers, P, rank, rows_cap, epoch, st);
    case FO_F16:
      return ce_shard_p2p_t<__half>(logits, target, loss_rows, lse, out_scalar, n_valid_out,
                                    dlogits, B, V_local, ld, v_offset, V, ignore_index,
                                    label_smoothing, reduction, peers, P, rank, rows_cap, epoch,
                                    st);
    default:
      return ce_shard_p2p_t<__nv_bfloat16>(logits, target, loss_rows, lse, out_scalar,
                                           n_valid_out, dlogits, B, V_local, ld, v_offset, V,
                                           ignore_index, label_smoothing, reduction, peers, P,
                                           rank, rows_cap, epoch, st);
  }
}

extern "C" int fo_ce_p2p_timeouts(unsigned int* count) {
  clear_error();
  FO_CHECK_ARG(count, "fo_ce_p2p_timeouts: null pointer");
  if (cudaMemcpyFromSymbol(count, g_ce_p2p_timeouts, sizeof(unsigned int)) != cudaSuccess) {
    set_error("fo_ce_p2p_timeouts: cannot read the device counter");
    return FO_ECUDA;
  }
  return FO_OK;
}
