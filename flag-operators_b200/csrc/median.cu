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


// ---------------------------------------------------------------------------
// row groups of RG warps (N <= 2048): keys in registers, one radix pass,
// compaction of the selected bucket, selection on the compacted list
// ---------------------------------------------------------------------------
// Element e of a row is held by warp w of the group, lane `lane`, slot (i, c):
//   e = ((i * RG + w) * 32 + lane) * VW + c
// (16-byte vectors when VW > 1).  The list holds composites
//   (key << 32) | index
// whose ascending order is the stable sort order, so the k-th composite is the
// answer without a separate tie rule.
template <int RG>
__device__ __forceinline__ void group_sync(int g) {
  if (RG == 1) __syncwarp();
  else asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(RG * 32) : "memory");
}

// Per-row-group scratch: CAP = elements per row group (list capacity), HW =
// histogram words (bins / 2, packed 16-bit counters).
// The histogram comes first and the struct is 16-byte aligned: the histogram
// is cleared with 16-byte stores (HW is a multiple of 4).
template <int RG, int CAP, int HW>
struct __align__(16) GroupSmem {
  static_assert(HW % 4 == 0, "histogram words must be a multiple of 4");
  uint32_t hist[HW];
  unsigned long long list[CAP];
  unsigned long long first_nan;
  uint32_t wsum[RG];
  uint32_t bucket, below, count, ncand;
};

// Finds the bin holding rank r among nbins bins (packed pairs in hist).
// Returns (bin, #elements in lower bins, #elements in bin) to every thread.
template <int RG, class GS>
__device__ __forceinline__ void group_find(GS& S, int g, int nbins, uint32_t r,
                                           uint32_t& bin, uint32_t& below, uint32_t& cnt) {
  const int t = threadIdx.x & (RG * 32 - 1);
  const int lane = t & 31, w = t >> 5;
  const int per = (nbins >> 1) / (RG * 32);  // words per thread (>= 1)
  const uint32_t* hw = S.hist + t * per;
  uint32_t tot = 0;
  for (int j = 0; j < per; ++j) tot += (hw[j] & 0xffffu) + (hw[j] >> 16);
  uint32_t inc = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += x;
  }
  if (RG > 1) {
    if (lane == 31) S.wsum[w] = inc;
    group_sync<RG>(g);
    uint32_t off = 0;
    for (int q = 0; q < w; ++q) off += S.wsum[q];
    inc += off;
  }
  const uint32_t exc = inc - tot;
  if (exc <= r && r < inc) {
    uint32_t acc = exc;
    for (int j = 0; j < per; ++j) {
      const uint32_t q = hw[j], c0 = q & 0xffffu, c1 = q >> 16;
      if (r < acc + c0) { S.bucket = 2 * (t * per + j); S.below = acc; S.count = c0; break; }
      acc += c0;
      if (r < acc + c1) { S.bucket = 2 * (t * per + j) + 1; S.below = acc; S.count = c1; break; }
      acc += c1;
    }
  }
  group_sync<RG>(g);
  bin = S.bucket;
  below = S.below;
  cnt = S.count;
}

template <int RG, class GS>
__device__ __forceinline__ void group_clear_hist(GS& S, int nbins) {
  const int t = threadIdx.x & (RG * 32 - 1);
  for (int j = t * 4; j < (nbins >> 1); j += RG * 32 * 4)
    *reinterpret_cast<uint4*>(S.hist + j) = make_uint4(0, 0, 0, 0);
}

__device__ __forceinline__ void hist_add(uint32_t* hist, uint32_t d) {
  atomicAdd(hist + (d >> 1), 1u << ((d & 1u) << 4));
}

template <int RG, int NI, int VW, int DIG0, int DIGL>
using GroupSmemOf = GroupSmem<RG, RG * 32 * NI * VW, (1 << (DIG0 > DIGL ? DIG0 : DIGL)) / 2>;

template <typename T, int RG, int NI, int VW, int DIG0, int DIGL, int GPC>
__global__ void __launch_bounds__(GPC * RG * 32, 3)
median_group_kernel(const T* __restrict__ x, T* __restrict__ vals, int64_t* __restrict__ idxs,
                    int64_t M, int N) {
  using Tr = KeyTraits<T>;
  using GS = GroupSmemOf<RG, NI, VW, DIG0, DIGL>;
  static_assert(sizeof(typename Tr::K) == 4, "32-bit keys only");
  extern __shared__ __align__(16) uint8_t median_smem[];
  const int g = threadIdx.x / (RG * 32);
  const int t = threadIdx.x & (RG * 32 - 1);
  const int lane = t & 31, w = t >> 5;
  GS& S = reinterpret_cast<GS*>(median_smem)[g];
  const int k = (N - 1) / 2;
  constexpr int SH0 = 32 - DIG0;

  // The next row's raw data is loaded into registers while the current row is
  // selected (rows are ~8 KiB; the load latency is otherwise exposed per row).
  constexpr int RN = VW > 1 ? 1 : VW;
  uint4 rv[NI];           // 16-byte vectors (VW > 1)
  T rs[NI][RN];           // scalars (VW == 1)
  auto load_row = [&](int64_t rrow) {
    if (rrow >= M) return;
    const T* xx = x + rrow * (int64_t)N;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int base = ((i * RG + w) * 32 + lane) * VW;
      if (VW > 1) {
        rv[i] = (base + VW <= N) ? ld_global_stream_v4(xx + base) : make_uint4(0, 0, 0, 0);
      } else {
#pragma unroll
        for (int c = 0; c < RN; ++c) rs[i][c] = (base + c < N) ? xx[base + c] : T(0);
      }
    }
  };
  const int64_t row0 = (int64_t)blockIdx.x * GPC + g;
  const int64_t rstep = (int64_t)gridDim.x * GPC;
  load_row(row0);

  for (int64_t row = row0; row < M; row += rstep) {
    const T* xr = x + row * (int64_t)N;
    uint32_t key[NI][VW];
    bool nan_seen = false;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int base = ((i * RG + w) * 32 + lane) * VW;
      if (VW > 1) {
        const T* e = reinterpret_cast<const T*>(&rv[i]);
#pragma unroll
        for (int c = 0; c < VW; ++c) {
          key[i][c] = Tr::key(e[c]);
          nan_seen |= (base + c < N) && Tr::isnan_(e[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < VW; ++c) {
          const T vv = rs[i][c < RN ? c : 0];
          key[i][c] = (base + c < N) ? Tr::key(vv) : 0u;
          nan_seen |= (base + c < N) && Tr::isnan_(vv);
        }
      }
    }
    load_row(row + rstep);
    if (t == 0) {
      S.first_nan = ~0ull;
      S.ncand = 0;
    }
    group_clear_hist<RG>(S, 1 << DIG0);
    group_sync<RG>(g);

    // ---- NaN: the first NaN in index order decides the row
    const bool any_nan = (RG == 1) ? __any_sync(0xffffffffu, nan_seen) : false;
    if (RG > 1 && nan_seen) atomicMin(&S.first_nan, 0ull);  // flag; resolved below
    if (RG > 1) group_sync<RG>(g);
    if ((RG == 1 && any_nan) || (RG > 1 && S.first_nan == 0ull)) {
      if (RG > 1) {
        group_sync<RG>(g);
        if (t == 0) S.first_nan = ~0ull;
        group_sync<RG>(g);
      }
      unsigned long long mine = ~0ull;
#pragma unroll
      for (int i = 0; i < NI; ++i)
#pragma unroll
        for (int c = 0; c < VW; ++c) {
          const int e = ((i * RG + w) * 32 + lane) * VW + c;
          if (e < N && Tr::isnan_(xr[e]) && (unsigned long long)e < mine) mine = e;
        }
      if (RG == 1) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const unsigned long long other = __shfl_xor_sync(0xffffffffu, mine, o);
          mine = other < mine ? other : mine;
        }
        if (lane == 0) S.first_nan = mine;
      } else if (mine != ~0ull) {
        atomicMin(&S.first_nan, mine);
      }
      group_sync<RG>(g);
      if (t == 0) {
        idxs[row] = (int64_t)S.first_nan;
        vals[row] = xr[S.first_nan];
      }
      group_sync<RG>(g);
      continue;
    }

    // ---- pass 0 over registers: top DIG0 bits
#pragma unroll
    for (int i = 0; i < NI; ++i)
#pragma unroll
      for (int c = 0; c < VW; ++c) {
        const int e = ((i * RG + w) * 32 + lane) * VW + c;
        if (e < N) hist_add(S.hist, key[i][c] >> SH0);
      }
    group_sync<RG>(g);
    uint32_t b0, below, cnt;
    group_find<RG>(S, g, 1 << DIG0, (uint32_t)k, b0, below, cnt);
    uint32_t r = (uint32_t)k - below;

    // ---- compact the bucket's elements as (key << 32 | index)
#pragma unroll
    for (int i = 0; i < NI; ++i)
#pragma unroll
      for (int c = 0; c < VW; ++c) {
        const int e = ((i * RG + w) * 32 + lane) * VW + c;
        if (e < N && (key[i][c] >> SH0) == b0) {
          const uint32_t pos = atomicAdd(&S.ncand, 1u);
          S.list[pos] = ((unsigned long long)key[i][c] << 32) | (uint32_t)e;
        }
      }
    group_sync<RG>(g);
    const uint32_t C = cnt;  // == S.ncand
    unsigned long long ans = 0;
    if (C <= 32) {
      // one warp: bitonic sort of <= 32 composites, pick the r-th
      if (w == 0) {
        unsigned long long v = lane < (int)C ? S.list[lane] : ~0ull;
#pragma unroll
        for (int kk = 2; kk <= 32; kk <<= 1) {
#pragma unroll
          for (int j = kk >> 1; j > 0; j >>= 1) {
            const unsigned long long o = __shfl_xor_sync(0xffffffffu, v, j);
            const bool up = ((lane & kk) == 0);
            const bool lower = ((lane & j) == 0);
            const unsigned long long mn = o < v ? o : v, mx = o < v ? v : o;
            v = (lower == up) ? mn : mx;
          }
        }
        ans = __shfl_sync(0xffffffffu, v, r);
        if (lane == 0) S.list[0] = ans;  // publish (list no longer needed)
      }
      group_sync<RG>(g);
      ans = S.list[0];
    } else {
      // radix passes over the list: remaining key bits, then the index bits
      // composite digit source: c = (key << 32) | idx; key bits [SH0-1 .. 0], idx bits [10..0]
      unsigned long long pref = 0, pmask = 0;
      const int nb_key = SH0;  // remaining key bits
      // pass plan over a virtual (nb_key + 11)-bit value v = (key & lowmask) << 11 | idx
      const int tot_bits = nb_key + 11;
      for (int done = 0; done < tot_bits;) {
        const int wbits = (tot_bits - done) < DIGL ? (tot_bits - done) : DIGL;
        const int sh = tot_bits - done - wbits;
        group_sync<RG>(g);
        group_clear_hist<RG>(S, 1 << DIGL);
        group_sync<RG>(g);
        for (uint32_t q = t; q < C; q += RG * 32) {
          const unsigned long long cpx = S.list[q];
          const unsigned long long vv =
              ((cpx >> 32) & ((1ull << nb_key) - 1ull)) << 11 | (cpx & 0x7ffull);
          if ((vv & pmask) == pref) hist_add(S.hist, (uint32_t)(vv >> sh) & ((1u << wbits) - 1u));
        }
        group_sync<RG>(g);
        uint32_t bb, bl, bc;
        group_find<RG>(S, g, 1 << DIGL, r, bb, bl, bc);
        r -= bl;
        pref |= (unsigned long long)bb << sh;
        pmask |= (unsigned long long)((1u << wbits) - 1u) << sh;
        done += wbits;
      }
      // pref now holds (remaining key bits, index)
      ans = ((unsigned long long)b0 << (32 + SH0)) | ((pref >> 11) << 32) | (pref & 0x7ffull);
    }
    if (t == 0) {
      int64_t e = (int64_t)(uint32_t)ans;
      if (e >= N) e = 0;  // unreachable; keeps the read in bounds
      idxs[row] = e;
      vals[row] = xr[e];
    }
    group_sync<RG>(g);
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
template <typename T, int RG, int NI, int VW, int DIG0>
int launch_group(const void* x, void* v, int64_t* idx, int64_t M, int N, cudaStream_t st) {
  constexpr int GPC = 8 / RG;                 // groups per CTA (256 threads)
  constexpr int DIGL = RG == 1 ? 8 : 11;      // digit width of the list passes
  auto kern = median_group_kernel<T, RG, NI, VW, DIG0, DIGL, GPC>;
  const int smem = (int)(GPC * sizeof(GroupSmemOf<RG, NI, VW, DIG0, DIGL>));
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
    set_error("median: cannot reserve %d bytes of shared memory", smem);
    return FO_ECUDA;
  }
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, GPC * RG * 32, smem);
  if (per_sm < 1) per_sm = 1;
  const int64_t need = (M + GPC - 1) / GPC;
  int64_t grid = (int64_t)num_sms() * per_sm;
  if (grid > need) grid = need;
  kern<<<(unsigned)grid, GPC * RG * 32, smem, st>>>((const T*)x, (T*)v, idx, M, N);
  return check_launch("median_group_kernel");
}

// Row length -> group width RG (warps), slots NI per lane, vector width VW.
template <typename T>
int dispatch_group(const void* x, void* v, int64_t* idx, int64_t M, int N, bool vec,
                   cudaStream_t st) {
  constexpr int VWV = 16 / sizeof(T);
  if (vec) {
    // 16-byte vectors: 32 * RG * NI * VWV >= N
    if (N <= 32 * VWV * 4) return launch_group<T, 1, 4, VWV, 8>(x, v, idx, M, N, st);
    if (N <= 64 * VWV * 4) return launch_group<T, 2, 4, VWV, 11>(x, v, idx, M, N, st);
    return launch_group<T, 4, 4, VWV, 11>(x, v, idx, M, N, st);
  }
  if (N <= 256) return launch_group<T, 1, 8, 1, 8>(x, v, idx, M, N, st);
  if (N <= 512) return launch_group<T, 1, 16, 1, 8>(x, v, idx, M, N, st);
  if (N <= 1024) return launch_group<T, 2, 16, 1, 11>(x, v, idx, M, N, st);
  return launch_group<T, 4, 16, 1, 11>(x, v, idx, M, N, st);
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
    const bool vec = aligned16(x) && ((N * (int64_t)sizeof(T)) % 16 == 0) && N >= 32 * VWV;
    return dispatch_group<T>(x, v, idx, M, (int)N, vec, st);
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
