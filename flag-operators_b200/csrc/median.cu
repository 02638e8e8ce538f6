// median along the last dimension (values + torch-compatible indices) and the
// global median, for sm_100a.
//
// Semantics: torch CPU median (the reference's CPU branch, operators/median.py:348-352):
//   k = (N - 1) / 2 (lower median); the index is the k-th entry of a STABLE
//   ascending sort (equal values keep index order); -0.0 == +0.0; a row holding
//   any NaN yields NaN and the index of its first NaN; the value returned is the
//   element stored at the index (bit-exact).
//
// Algorithm: radix select on an order-preserving unsigned key
//   float: key = bits ^ (sign ? 0xffffffff : 0x80000000) after -0.0 -> +0.0
//   int:   key = bits ^ sign bit
// in digits of 11 bits from the most significant end.  Each pass histograms the
// digit of the elements whose higher digits equal the prefix selected so far and
// picks the bucket holding rank r.  After the last pass the key K of the k-th
// element is known, and r is its occurrence rank among the elements equal to K;
// the answer is the r-th such element in index order, found with ballots.
//
// Short rows (N <= 2048): one warp per row.  The row sits in registers (loaded
// once, 16-byte vectors when the row is 16-byte aligned), the histogram is
// private to the warp in shared memory as packed 16-bit counters, and no block
// barrier is needed.  Long rows and the global median: one CTA per row, passes
// re-read the row (L2 hits for rows that fit in L2).
#include "common.cuh"

namespace fo {
namespace {

// ---------------------------------------------------------------------------
// keys
// ---------------------------------------------------------------------------
template <typename T> struct KeyTraits;
template <> struct KeyTraits<float> {
  using K = uint32_t;
  static __device__ __forceinline__ K key(float x) {
    const uint32_t u = __float_as_uint(__fadd_rn(x, 0.0f));  // -0.0 + 0.0 = +0.0
    return u ^ ((uint32_t)((int32_t)u >> 31) | 0x80000000u);
  }
  static __device__ __forceinline__ bool isnan_(float x) { return x != x; }
};
template <> struct KeyTraits<__half> {
  using K = uint32_t;
  static __device__ __forceinline__ K key(__half x) { return KeyTraits<float>::key(__half2float(x)); }
  static __device__ __forceinline__ bool isnan_(__half x) { return __hisnan(x); }
};
template <> struct KeyTraits<__nv_bfloat16> {
  using K = uint32_t;
  static __device__ __forceinline__ K key(__nv_bfloat16 x) {
    return KeyTraits<float>::key(__bfloat162float(x));
  }
  static __device__ __forceinline__ bool isnan_(__nv_bfloat16 x) { return __hisnan(x); }
};
template <> struct KeyTraits<int32_t> {
  using K = uint32_t;
  static __device__ __forceinline__ K key(int32_t x) { return (uint32_t)x ^ 0x80000000u; }
  static __device__ __forceinline__ bool isnan_(int32_t) { return false; }
};
template <> struct KeyTraits<int64_t> {
  using K = uint64_t;
  static __device__ __forceinline__ K key(int64_t x) { return (uint64_t)x ^ 0x8000000000000000ull; }
  static __device__ __forceinline__ bool isnan_(int64_t) { return false; }
};

template <typename K> struct Digits {
  static constexpr int kBits = 8 * sizeof(K);
  static constexpr int kPasses = (kBits + 10) / 11;
  static __device__ __forceinline__ int shift(int p) {
    const int s = kBits - 11 * (p + 1);
    return s > 0 ? s : 0;
  }
  static __device__ __forceinline__ int width(int p) { return kBits - 11 * p - shift(p); }
};

constexpr int kWarpHistWords = 1024;  // 2048 bins as packed 16-bit pairs

// ---------------------------------------------------------------------------
// warp per row
// ---------------------------------------------------------------------------
// Lane `lane` holds, for i < NI and c < VW, the element at index
// i * 32 * VW + lane * VW + c; index order is therefore (i, lane, c).
template <typename T, int NI, int VW, int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
median_warp_kernel(const T* __restrict__ x, T* __restrict__ vals, int64_t* __restrict__ idxs,
                   int64_t M, int N) {
  using Tr = KeyTraits<T>;
  using K = typename Tr::K;
  using D = Digits<K>;
  __shared__ uint32_t hist_all[WARPS][kWarpHistWords];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  uint32_t* hist = hist_all[wid];
  const int64_t gw = (int64_t)blockIdx.x * WARPS + wid;
  const int64_t nwarps = (int64_t)gridDim.x * WARPS;
  const int k = (N - 1) / 2;

  for (int64_t row = gw; row < M; row += nwarps) {
    const T* xr = x + row * (int64_t)N;
    K key[NI][VW];
    bool nan_seen = false;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int base = i * 32 * VW + lane * VW;
      if (VW > 1 && base + VW <= N) {
        uint4 u = ld_global_stream_v4(xr + base);
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int c = 0; c < VW; ++c) {
          key[i][c] = Tr::key(e[c]);
          nan_seen |= Tr::isnan_(e[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < VW; ++c) {
          if (base + c < N) {
            const T v = xr[base + c];
            key[i][c] = Tr::key(v);
            nan_seen |= Tr::isnan_(v);
          } else {
            key[i][c] = 0;
          }
        }
      }
    }

    int found_i = -1, found_c = 0, found_lane = 0;
    if (__any_sync(0xffffffffu, nan_seen)) {
      // first NaN in index order
      for (int i = 0; i < NI && found_i < 0; ++i) {
        int lane_c = VW;
#pragma unroll
        for (int c = VW - 1; c >= 0; --c) {
          const int pos = i * 32 * VW + lane * VW + c;
          if (pos < N && Tr::isnan_(xr[pos])) lane_c = c;
        }
        const uint32_t m = __ballot_sync(0xffffffffu, lane_c < VW);
        if (m) {
          found_lane = __ffs(m) - 1;
          found_c = __shfl_sync(0xffffffffu, lane_c, found_lane);
          found_i = i;
        }
      }
    } else {
      K prefix = 0, pmask = 0;
      int r = k;
#pragma unroll 1
      for (int p = 0; p < D::kPasses; ++p) {
        const int sh = D::shift(p);
        const int w = D::width(p);
        const uint32_t dmask = (1u << w) - 1u;
        const int words = (1 << w) >> 1;
        for (int j = lane * 4; j < words; j += 128)
          *reinterpret_cast<uint4*>(hist + j) = make_uint4(0, 0, 0, 0);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < NI; ++i) {
#pragma unroll
          for (int c = 0; c < VW; ++c) {
            const int pos = i * 32 * VW + lane * VW + c;
            const bool mine = pos < N && (key[i][c] & pmask) == prefix;
            if (p == 0) {
              if (mine) {
                const uint32_t d = (uint32_t)(key[i][c] >> sh) & dmask;
                atomicAdd(hist + (d >> 1), 1u << ((d & 1u) << 4));
              }
            } else if (__any_sync(0xffffffffu, mine)) {
              if (mine) {
                const uint32_t d = (uint32_t)(key[i][c] >> sh) & dmask;
                atomicAdd(hist + (d >> 1), 1u << ((d & 1u) << 4));
              }
            }
          }
        }
        __syncwarp();
        // bucket holding rank r: lane sums its 1/32 slice of the words
        const int per = words >> 5;  // words per lane (>= 16 when w >= 10)
        uint32_t tot = 0;
        for (int j = 0; j < per; j += 4) {
          const uint4 q = *reinterpret_cast<const uint4*>(hist + lane * per + j);
          tot += (q.x & 0xffffu) + (q.x >> 16) + (q.y & 0xffffu) + (q.y >> 16) + (q.z & 0xffffu) +
                 (q.z >> 16) + (q.w & 0xffffu) + (q.w >> 16);
        }
        uint32_t inc = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
          if (lane >= o) inc += t;
        }
        const uint32_t exc = inc - tot;
        const uint32_t sel = __ballot_sync(0xffffffffu, exc <= (uint32_t)r && (uint32_t)r < inc);
        const int L = __ffs(sel) - 1;
        const uint32_t base_cnt = __shfl_sync(0xffffffffu, exc, L);
        // inside lane L's slice: per words, each lane takes per/32 words
        uint32_t bucket = 0, below = 0;
        {
          const int wpl = per >> 5 > 0 ? per >> 5 : 1;  // words per lane in the slice
          const int w0 = L * per + lane * wpl;
          uint32_t cnt = 0;
          if (lane * wpl < per)
            for (int j = 0; j < wpl; ++j) {
              const uint32_t q = hist[w0 + j];
              cnt += (q & 0xffffu) + (q >> 16);
            }
          uint32_t inc2 = cnt;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, inc2, o);
            if (lane >= o) inc2 += t;
          }
          const uint32_t exc2 = base_cnt + inc2 - cnt;
          const bool here = lane * wpl < per && exc2 <= (uint32_t)r && (uint32_t)r < exc2 + cnt;
          const uint32_t sel2 = __ballot_sync(0xffffffffu, here);
          const int L2 = __ffs(sel2) - 1;
          if (lane == L2) {
            uint32_t acc = exc2;
            for (int j = 0; j < wpl; ++j) {
              const uint32_t q = hist[w0 + j];
              const uint32_t c0 = q & 0xffffu, c1 = q >> 16;
              const uint32_t word = (uint32_t)(w0 + j);
              if ((uint32_t)r < acc + c0) { bucket = word * 2; below = acc; break; }
              acc += c0;
              if ((uint32_t)r < acc + c1) { bucket = word * 2 + 1; below = acc; break; }
              acc += c1;
            }
          }
          bucket = __shfl_sync(0xffffffffu, bucket, L2);
          below = __shfl_sync(0xffffffffu, below, L2);
        }
        r -= (int)below;
        prefix |= (K)bucket << sh;
        pmask |= (K)dmask << sh;
        __syncwarp();
      }
      // r-th occurrence (index order) of key == prefix.  Fully unrolled so the
      // key array stays in registers.
      int cnt[NI];
      int fi = -1;
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        int c_i = 0;
#pragma unroll
        for (int c = 0; c < VW; ++c) {
          const int pos = i * 32 * VW + lane * VW + c;
          c_i += (pos < N && key[i][c] == prefix) ? 1 : 0;
        }
        cnt[i] = c_i;
        const int total = (int)__reduce_add_sync(0xffffffffu, (unsigned)c_i);
        if (fi < 0) {
          if (r < total) fi = i;
          else r -= total;
        }
      }
      int my = 0;
#pragma unroll
      for (int i = 0; i < NI; ++i) my = (i == fi) ? cnt[i] : my;
      int inc = my;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
      }
      const int exc = inc - my;
      const uint32_t sel = __ballot_sync(0xffffffffu, fi >= 0 && exc <= r && r < inc);
      found_lane = sel ? __ffs(sel) - 1 : 0;
      int cc = 0, rr = r - exc;
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        if (i == fi) {
#pragma unroll
          for (int c = 0; c < VW; ++c) {
            const int pos = i * 32 * VW + lane * VW + c;
            if (pos < N && key[i][c] == prefix) {
              if (rr == 0) cc = c;
              --rr;
            }
          }
        }
      }
      found_c = __shfl_sync(0xffffffffu, cc, found_lane);
      found_i = fi;
    }
    if (lane == 0) {
      int64_t pos = (int64_t)found_i * 32 * VW + found_lane * VW + found_c;
      if (found_i < 0 || pos >= N) pos = 0;  // unreachable; keeps the read in bounds
      idxs[row] = pos;
      vals[row] = xr[pos];
    }
  }
}

// ---------------------------------------------------------------------------
// CTA per row (any N; also the global median)
// ---------------------------------------------------------------------------
constexpr int kCtaThreads = 512;

template <typename T>
__global__ void __launch_bounds__(kCtaThreads)
median_cta_kernel(const T* __restrict__ x, T* __restrict__ vals, int64_t* __restrict__ idxs,
                  int64_t M, int64_t N) {
  using Tr = KeyTraits<T>;
  using K = typename Tr::K;
  using D = Digits<K>;
  __shared__ uint32_t hist[2048];
  __shared__ uint32_t wsum[kCtaThreads / 32];
  __shared__ unsigned long long s_first_nan;
  __shared__ uint32_t s_bucket, s_below;
  __shared__ int64_t s_found;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  constexpr int NW = kCtaThreads / 32;
  const int64_t k = (N - 1) / 2;

  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const T* xr = x + row * N;
    if (tid == 0) {
      s_first_nan = ~0ull;
      s_found = 0;
      s_bucket = 0;
      s_below = 0;
    }
    __syncthreads();
    int64_t my_nan = -1;
    for (int64_t j = tid; j < N; j += kCtaThreads)
      if (Tr::isnan_(xr[j])) { my_nan = j; break; }
    if (my_nan >= 0) atomicMin(&s_first_nan, (unsigned long long)my_nan);
    __syncthreads();
    if (s_first_nan != ~0ull) {
      if (tid == 0) {
        idxs[row] = (int64_t)s_first_nan;
        vals[row] = xr[s_first_nan];
      }
      __syncthreads();
      continue;
    }
    K prefix = 0, pmask = 0;
    int64_t r = k;
    for (int p = 0; p < D::kPasses; ++p) {
      const int sh = D::shift(p), w = D::width(p);
      const uint32_t nb = 1u << w, dmask = nb - 1u;
      for (uint32_t j = tid; j < nb; j += kCtaThreads) hist[j] = 0;
      __syncthreads();
      for (int64_t j = tid; j < N; j += kCtaThreads) {
        const K kk = Tr::key(xr[j]);
        if ((kk & pmask) == prefix) atomicAdd(hist + ((uint32_t)(kk >> sh) & dmask), 1u);
      }
      __syncthreads();
      // each thread owns nb / kCtaThreads consecutive bins
      const uint32_t per = (nb + kCtaThreads - 1) / kCtaThreads;
      uint32_t cnt = 0;
      for (uint32_t j = 0; j < per; ++j) {
        const uint32_t b = tid * per + j;
        if (b < nb) cnt += hist[b];
      }
      uint32_t inc = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
      }
      if (lane == 31) wsum[wid] = inc;
      __syncthreads();
      uint32_t woff = 0;
      for (int q = 0; q < wid; ++q) woff += wsum[q];
      const uint32_t exc = woff + inc - cnt;
      if ((uint64_t)exc <= (uint64_t)r && (uint64_t)r < (uint64_t)exc + cnt) {
        uint32_t acc = exc;
        for (uint32_t j = 0; j < per; ++j) {
          const uint32_t b = tid * per + j;
          const uint32_t c = b < nb ? hist[b] : 0;
          if ((uint64_t)r < (uint64_t)acc + c) { s_bucket = b; s_below = acc; break; }
          acc += c;
        }
      }
      __syncthreads();
      r -= s_below;
      prefix |= (K)s_bucket << sh;
      pmask |= (K)dmask << sh;
      __syncthreads();
    }
    // r-th occurrence of key == prefix: thread t scans the contiguous range
    // [t*chunk, (t+1)*chunk), so occurrences are ordered by thread.
    const int64_t chunk = (N + kCtaThreads - 1) / kCtaThreads;
    const int64_t j0 = (int64_t)tid * chunk;
    const int64_t j1 = j0 + chunk < N ? j0 + chunk : N;
    uint32_t cnt = 0;
    for (int64_t j = j0; j < j1; ++j) cnt += (Tr::key(xr[j]) == prefix) ? 1u : 0u;
    uint32_t inc = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += t;
    }
    __syncthreads();
    if (lane == 31) wsum[wid] = inc;
    __syncthreads();
    uint32_t woff = 0;
    for (int q = 0; q < wid; ++q) woff += wsum[q];
    const uint32_t exc = woff + inc - cnt;
    if ((uint64_t)exc <= (uint64_t)r && (uint64_t)r < (uint64_t)exc + cnt) {
      int64_t rr = r - exc;
      for (int64_t j = j0; j < j1; ++j) {
        if (Tr::key(xr[j]) == prefix) {
          if (rr == 0) { s_found = j; break; }
          --rr;
        }
      }
    }
    __syncthreads();
    if (tid == 0) {
      idxs[row] = s_found;
      vals[row] = xr[s_found];
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// dispatch
// ---------------------------------------------------------------------------
template <typename T, int NI, int VW>
int launch_warp(const void* x, void* v, int64_t* idx, int64_t M, int N, cudaStream_t st) {
  constexpr int WARPS = 8;
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, median_warp_kernel<T, NI, VW, WARPS>,
                                                WARPS * 32, 0);
  if (per_sm < 1) per_sm = 1;
  int64_t need = (M + WARPS - 1) / WARPS;
  int64_t grid = (int64_t)num_sms() * per_sm;
  if (grid > need) grid = need;
  median_warp_kernel<T, NI, VW, WARPS><<<(unsigned)grid, WARPS * 32, 0, st>>>(
      (const T*)x, (T*)v, idx, M, N);
  return check_launch("median_warp_kernel");
}

template <typename T, int VW>
int pick_ni(const void* x, void* v, int64_t* idx, int64_t M, int N, cudaStream_t st) {
  const int ni = (N + 32 * VW - 1) / (32 * VW);
  if (ni <= 1) return launch_warp<T, 1, VW>(x, v, idx, M, N, st);
  if (ni <= 2) return launch_warp<T, 2, VW>(x, v, idx, M, N, st);
  if (ni <= 4) return launch_warp<T, 4, VW>(x, v, idx, M, N, st);
  if (ni <= 8) return launch_warp<T, 8, VW>(x, v, idx, M, N, st);
  if (ni <= 16) return launch_warp<T, 16, VW>(x, v, idx, M, N, st);
  if (VW == 1 && ni <= 32) return launch_warp<T, 32, 1>(x, v, idx, M, N, st);
  return launch_warp<T, 64, 1>(x, v, idx, M, N, st);
}

template <typename T>
int launch_cta(const void* x, void* v, int64_t* idx, int64_t M, int64_t N, cudaStream_t st) {
  int64_t grid = (int64_t)num_sms() * 4;
  if (grid > M) grid = M;
  median_cta_kernel<T><<<(unsigned)grid, kCtaThreads, 0, st>>>((const T*)x, (T*)v, idx, M, N);
  return check_launch("median_cta_kernel");
}

template <typename T>
int median_dim_t(const void* x, void* v, int64_t* idx, int64_t M, int64_t N, cudaStream_t st) {
  if (sizeof(T) <= 4 && N <= 2048) {
    constexpr int VWV = 16 / (sizeof(T) <= 4 ? sizeof(T) : 4);
    const bool vec = aligned16(x) && ((N * (int64_t)sizeof(T)) % 16 == 0);
    if (vec && N >= 32 * VWV) return pick_ni<T, VWV>(x, v, idx, M, (int)N, st);
    return pick_ni<T, 1>(x, v, idx, M, (int)N, st);
  }
  return launch_cta<T>(x, v, idx, M, N, st);
}

}  // namespace
}  // namespace fo

using namespace fo;

extern "C" int fo_median_dim(const void* x, void* values, int64_t* indices, int64_t M, int64_t N,
                             int dtype, void* stream) {
  clear_error();
  FO_CHECK_ARG(M >= 0 && N >= 0, "median: negative size");
  if (M == 0) return FO_OK;
  FO_CHECK_ARG(N > 0, "median: cannot compute the median of an empty dimension");
  FO_CHECK_ARG(x && values && indices, "median: null pointer");
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case FO_F32: return median_dim_t<float>(x, values, indices, M, N, st);
    case FO_F16: return median_dim_t<__half>(x, values, indices, M, N, st);
    case FO_BF16: return median_dim_t<__nv_bfloat16>(x, values, indices, M, N, st);
    case FO_I32: return median_dim_t<int32_t>(x, values, indices, M, N, st);
    case FO_I64: return launch_cta<int64_t>(x, values, indices, M, N, st);
  }
  set_error("median: unsupported dtype code %d", dtype);
  return FO_EDTYPE;
}

extern "C" int fo_median_all_workspace_bytes(int64_t n, int64_t* bytes) {
  clear_error();
  FO_CHECK_ARG(bytes && n >= 0, "fo_median_all_workspace_bytes: bad argument");
  *bytes = 8;  // the index of the selected element
  return FO_OK;
}

extern "C" int fo_median_all(const void* x, void* value, int64_t n, int dtype, void* workspace,
                             int64_t ws_bytes, void* stream) {
  clear_error();
  FO_CHECK_ARG(n > 0, "median() input must not be empty");
  FO_CHECK_ARG(x && value, "median: null pointer");
  if (!workspace || ws_bytes < 8) {
    set_error("median: workspace of 8 bytes required");
    return FO_EWORKSPACE;
  }
  cudaStream_t st = as_stream(stream);
  int64_t* idx = reinterpret_cast<int64_t*>(workspace);
  switch (dtype) {
    case FO_F32: return launch_cta<float>(x, value, idx, 1, n, st);
    case FO_F16: return launch_cta<__half>(x, value, idx, 1, n, st);
    case FO_BF16: return launch_cta<__nv_bfloat16>(x, value, idx, 1, n, st);
    case FO_I32: return launch_cta<int32_t>(x, value, idx, 1, n, st);
    case FO_I64: return launch_cta<int64_t>(x, value, idx, 1, n, st);
  }
  set_error("median: unsupported dtype code %d", dtype);
  return FO_EDTYPE;
}
