// scatter_reduce (sum, prod, mean, amax, amin; include_self) for sm_100a.
//
// Semantics: torch.Tensor.scatter_reduce_ on CPU (the reference's CPU branch,
// operators/scatter_reduce.py:397-398, 427-429, 457-459):
//   for every position p of index: out[p with p[dim] := index[p]] op= src[p]
//   include_self=False: a cell reached by >= 1 index takes the reduction of its
//     src values only; cells never reached keep self.
//   mean: sum / count (count includes self when include_self); integer mean
//     rounds toward -inf.  amax/amin propagate NaN.
//
// Design.
//  * One pass over (index, src): 16-byte vector loads on the contiguous 1-D
//    path, generic strided addressing for 2-4-D.
//  * Each CTA keeps a shared-memory cache of output cells (hashed slots, tag =
//    output offset).  An update whose cell owns a slot is a shared-memory
//    atomic; others go straight to global atomics (L2).  At the end the CTA
//    flushes its slots with one global atomic each.  Skewed (Zipf) indices —
//    thousands of updates on a few cells — thus cost shared-memory atomics
//    instead of serialised same-address L2 atomics; uniform indices pass
//    through with one extra shared-memory probe.
//  * Float amax/amin reduce order-preserving uint32 keys with native integer
//    atomicMax/Min (no CAS loop); NaN maps to the extreme key so it wins.
//    prod is the only CAS loop.
//  * Float sum without self and float mean accumulate (sum, count) pairs in
//    one interleaved scratch with a single 8-byte vector reduction
//    (red.global.add.v2.f32) per update instead of two atomics; counts held
//    as floats are exact while a call has at most 2^24 updates (else separate
//    int32 counts).
//  * The contiguous 1-D pass is software-pipelined: the next quad's index and
//    src loads are in flight while the current quad's updates are issued.
//  * A scratch accumulator (+ int32 counts) is used only when needed:
//    include_self=False (to know which cells were reached), mean (counts),
//    float amax/amin (keys) and 16-bit floats (fp32 accumulation).  Then an
//    init pass and a finalize pass run over the output (1/16 of the traffic of
//    the scatter pass at the benchmark shape).
#include <limits.h>

#include "common.cuh"

namespace fo {
namespace {

enum Op { kSum = FO_SUM, kProd = FO_PROD, kMean = FO_MEAN, kAmax = FO_AMAX, kAmin = FO_AMIN };

constexpr int kThreads = 512;
template <typename A> struct Slots { static constexpr int kLog = sizeof(A) == 8 ? 11 : 12; static constexpr int kN = 1 << kLog; };
constexpr uint32_t kEmpty = 0xffffffffu;

// ---------------------------------------------------------------------------
// value <-> accumulator conversions
// ---------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float tof(T v) { return to_f<T>(v); }
template <> __device__ __forceinline__ float tof<int32_t>(int32_t v) { return (float)v; }
template <> __device__ __forceinline__ float tof<int64_t>(int64_t v) { return (float)v; }

__device__ __forceinline__ uint32_t fkey(float x, bool nan_high) {
  if (x != x) return nan_high ? 0xffffffffu : 0u;
  const uint32_t u = __float_as_uint(x);
  return u ^ ((uint32_t)((int32_t)u >> 31) | 0x80000000u);
}
__device__ __forceinline__ float funkey(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k ^ 0x80000000u) : ~k;
  return __uint_as_float(u);
}

// Accumulator traits: A is the type atomics operate on.
template <typename T, int OP, bool KEYS> struct Acc;

// float amax/amin through keys
template <typename T, int OP> struct Acc<T, OP, true> {
  using A = uint32_t;
  static __device__ __forceinline__ A identity() { return OP == kAmax ? 0u : 0xffffffffu; }
  static __device__ __forceinline__ A from(T v) { return fkey(tof<T>(v), OP == kAmax); }
  static __device__ __forceinline__ void op(A* p, A v) {
    if (OP == kAmax) atomicMax(p, v);
    else atomicMin(p, v);
  }
  static __device__ __forceinline__ A comb(A a, A b) { return OP == kAmax ? max(a, b) : min(a, b); }
};

template <typename A> __device__ __forceinline__ void atomic_add_a(A* p, A v);
template <> __device__ __forceinline__ void atomic_add_a<float>(float* p, float v) { atomicAdd(p, v); }
template <> __device__ __forceinline__ void atomic_add_a<int32_t>(int32_t* p, int32_t v) { atomicAdd(p, v); }
template <> __device__ __forceinline__ void atomic_add_a<int64_t>(int64_t* p, int64_t v) {
  atomicAdd(reinterpret_cast<unsigned long long*>(p), (unsigned long long)v);
}
template <typename A> __device__ __forceinline__ void atomic_mul_a(A* p, A v);
template <> __device__ __forceinline__ void atomic_mul_a<float>(float* p, float v) {
  unsigned int* q = reinterpret_cast<unsigned int*>(p);
  unsigned int old = *reinterpret_cast<volatile unsigned int*>(q), assumed;
  do {
    assumed = old;
    old = atomicCAS(q, assumed, __float_as_uint(__uint_as_float(assumed) * v));
  } while (old != assumed);
}
template <> __device__ __forceinline__ void atomic_mul_a<int32_t>(int32_t* p, int32_t v) {
  int old = *reinterpret_cast<volatile int*>(p), assumed;
  do {
    assumed = old;
    old = atomicCAS(p, assumed, (int)((uint32_t)assumed * (uint32_t)v));
  } while (old != assumed);
}
template <> __device__ __forceinline__ void atomic_mul_a<int64_t>(int64_t* p, int64_t v) {
  unsigned long long* q = reinterpret_cast<unsigned long long*>(p);
  unsigned long long old = *reinterpret_cast<volatile unsigned long long*>(q), assumed;
  do {
    assumed = old;
    old = atomicCAS(q, assumed, (unsigned long long)((uint64_t)assumed * (uint64_t)v));
  } while (old != assumed);
}
__device__ __forceinline__ void atomic_max_a(int32_t* p, int32_t v) { atomicMax(p, v); }
__device__ __forceinline__ void atomic_min_a(int32_t* p, int32_t v) { atomicMin(p, v); }
__device__ __forceinline__ void atomic_max_a(int64_t* p, int64_t v) {
  atomicMax(reinterpret_cast<long long*>(p), (long long)v);
}
__device__ __forceinline__ void atomic_min_a(int64_t* p, int64_t v) {
  atomicMin(reinterpret_cast<long long*>(p), (long long)v);
}

// (sum, count) pair update: one 8-byte vector reduction in L2
__device__ __forceinline__ void red_pair(float* p, float v, float c) {
  asm volatile("red.relaxed.gpu.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(v), "f"(c)
               : "memory");
}

template <typename T> struct AccType { using A = T; };
template <> struct AccType<__half> { using A = float; };
template <> struct AccType<__nv_bfloat16> { using A = float; };

template <typename T, int OP> struct Acc<T, OP, false> {
  using A = typename AccType<T>::A;
  static __device__ __forceinline__ A identity() {
    if (OP == kProd) return (A)1;
    if (OP == kAmax) return sizeof(A) == 8 ? (A)LLONG_MIN : (A)INT_MIN;
    if (OP == kAmin) return sizeof(A) == 8 ? (A)LLONG_MAX : (A)INT_MAX;
    return (A)0;
  }
  static __device__ __forceinline__ A from(T v);
  static __device__ __forceinline__ void op(A* p, A v) {
    if (OP == kSum || OP == kMean) atomic_add_a<A>(p, v);
    else if (OP == kProd) atomic_mul_a<A>(p, v);
    else if constexpr (sizeof(A) == 4 && !std::is_same<A, float>::value) {
      if (OP == kAmax) atomic_max_a((int32_t*)p, (int32_t)v);
      else atomic_min_a((int32_t*)p, (int32_t)v);
    } else if constexpr (sizeof(A) == 8) {
      if (OP == kAmax) atomic_max_a((int64_t*)p, (int64_t)v);
      else atomic_min_a((int64_t*)p, (int64_t)v);
    }
  }
  // the same reduction of two values (warp aggregation before an atomic)
  static __device__ __forceinline__ A comb(A a, A b) {
    if (OP == kSum || OP == kMean) return a + b;
    if (OP == kProd) return a * b;
    if (OP == kAmax) return a > b ? a : b;
    return a < b ? a : b;
  }
};

// One compare-and-swap step of a product update: returns the cell's old value
// and sets ok when it equalled `assumed` (bitwise), i.e. the product was stored.
__device__ __forceinline__ float cas_mul(float* p, float assumed, float v, bool& ok) {
  const unsigned int a = __float_as_uint(assumed);
  const unsigned int o =
      atomicCAS(reinterpret_cast<unsigned int*>(p), a, __float_as_uint(assumed * v));
  ok = (o == a);
  return __uint_as_float(o);
}
__device__ __forceinline__ int32_t cas_mul(int32_t* p, int32_t assumed, int32_t v, bool& ok) {
  const int o = atomicCAS(p, assumed, (int)((uint32_t)assumed * (uint32_t)v));
  ok = (o == assumed);
  return o;
}
__device__ __forceinline__ int64_t cas_mul(int64_t* p, int64_t assumed, int64_t v, bool& ok) {
  const unsigned long long a = (unsigned long long)assumed;
  const unsigned long long o = atomicCAS(reinterpret_cast<unsigned long long*>(p), a,
                                         (unsigned long long)((uint64_t)assumed * (uint64_t)v));
  ok = (o == a);
  return (int64_t)o;
}
template <typename T, int OP>
__device__ __forceinline__ typename Acc<T, OP, false>::A Acc<T, OP, false>::from(T v) {
  if constexpr (std::is_same<A, float>::value) return tof<T>(v);
  else return (A)v;
}

// ---------------------------------------------------------------------------
// the scatter pass
// ---------------------------------------------------------------------------
struct Geo {
  int64_t shape[4];    // index shape (padded with 1)
  int64_t istr[4];     // index strides
  int64_t sstr[4];     // src strides
  int64_t ostr[4];     // out strides
  int64_t out_dim;     // out.shape[dim]
  int dim;
  int ndim;
};

// PAIR: acc holds interleaved (sum, count) floats and cnt is unused.
template <typename T, typename I, int OP, bool KEYS, bool CNT, bool PAIR, int NDIM, bool VEC>
__global__ void __launch_bounds__(kThreads)
scatter_kernel(const T* __restrict__ src, const I* __restrict__ index,
               typename Acc<T, OP, KEYS>::A* __restrict__ acc, int32_t* __restrict__ cnt,
               int64_t n, Geo g, int32_t* __restrict__ err, bool use_cache) {
  using AT = Acc<T, OP, KEYS>;
  using A = typename AT::A;
  constexpr int kSlots = Slots<A>::kN;
  __shared__ uint32_t s_tag[kSlots];
  __shared__ A s_val[kSlots];
  constexpr bool kCnt = CNT || PAIR;
  __shared__ int32_t s_cnt[kCnt ? kSlots : 1];
  if (use_cache) {
    for (int j = threadIdx.x; j < kSlots; j += blockDim.x) {
      s_tag[j] = kEmpty;
      s_val[j] = AT::identity();
      if (kCnt) s_cnt[j] = 0;
    }
    __syncthreads();
  }
  int32_t bad = 0;

  // c: how many updates v stands for (warp-aggregated updates carry c > 1)
  auto cache_update = [&](int64_t off, A v, int c) -> bool {
    const uint32_t o32 = (uint32_t)off;
    const uint32_t slot = (o32 * 2654435761u) >> (32 - Slots<A>::kLog);
    uint32_t t = s_tag[slot];
    if (t == kEmpty) {
      const uint32_t prev = atomicCAS(&s_tag[slot], kEmpty, o32);
      t = (prev == kEmpty) ? o32 : prev;
    }
    if (t != o32) return false;
    AT::op(&s_val[slot], v);
    if (kCnt) atomicAdd(&s_cnt[slot], c);
    return true;
  };
  auto global_update = [&](int64_t off, A v, int c) {
    if constexpr (PAIR) {
      red_pair(reinterpret_cast<float*>(acc) + 2 * off, (float)v, (float)c);
    } else {
      AT::op(acc + off, v);
      if (CNT) atomicAdd(cnt + off, c);
    }
  };
  auto update = [&](int64_t off, A v) {
    if (use_cache && cache_update(off, v, 1)) return;
    global_update(off, v, 1);
  };

  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (VEC) {
    // 1-D, contiguous index (int64) and src, 16-byte aligned: quads of 4
    // elements, grid-strided; the next quad is loaded while this one updates
    static_assert(!VEC || sizeof(I) == 8, "vector path expects int64 index");
    const int64_t nq = n / 4;
    struct Quad {
      uint4 i01, i23;
      T sv[4];
    };
    auto load_quad = [&](int64_t q, Quad& Q) {
      if (q >= nq) return;
      Q.i01 = ld_global_stream_v4(index + q * 4);
      Q.i23 = ld_global_stream_v4(index + q * 4 + 2);
      if constexpr (sizeof(T) == 4) {
        const uint4 s4 = ld_global_stream_v4(src + q * 4);
        memcpy(Q.sv, &s4, 16);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) Q.sv[e] = src[q * 4 + e];
      }
    };
    // Every lane of a warp runs the same iterations (lanes past the end pass
    // valid = false), so the warp can aggregate: lanes whose updates hit one
    // cell are found with match.any; the lowest of them combines the others'
    // values and issues one update carrying their count.  With skewed indices
    // this turns several same-address atomics into one.  A warp keeps
    // aggregating only if its first quad held at least 4 such duplicates
    // (match.any costs more than it saves on spread-out indices).  Products
    // that reach global memory are issued as a batch of independent
    // compare-and-swaps.
    const int lane = threadIdx.x & 31;
    bool agg = use_cache, probing = use_cache;
    auto do_quad = [&](const Quad& Q, bool valid) {
      int64_t iv[4];
      iv[0] = (int64_t)(((uint64_t)Q.i01.y << 32) | Q.i01.x);
      iv[1] = (int64_t)(((uint64_t)Q.i01.w << 32) | Q.i01.z);
      iv[2] = (int64_t)(((uint64_t)Q.i23.y << 32) | Q.i23.x);
      iv[3] = (int64_t)(((uint64_t)Q.i23.w << 32) | Q.i23.z);
      int64_t off[4];
      A val[4];
      bool go[4];
      int dups = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        bool act = valid;
        if (act && (iv[e] < 0 || iv[e] >= g.out_dim)) {
          ++bad;
          act = false;
        }
        off[e] = iv[e] * g.ostr[0];
        A v = valid ? AT::from(Q.sv[e]) : AT::identity();
        int c = 1;
        if (agg) {  // warp-uniform; offsets fit 32 bits and never equal the sentinel
          const uint32_t peers =
              __match_any_sync(0xffffffffu, act ? (uint32_t)off[e] : 0xffffffffu);
          const int lead = __ffs(peers) - 1;
          const bool follower = act && lane != lead;
          uint32_t fol = __ballot_sync(0xffffffffu, follower);
          dups += __popc(fol);
          while (fol) {  // warp-uniform: one shuffle per follower lane
            const int src = __ffs(fol) - 1;
            fol &= fol - 1;
            const A ov = __shfl_sync(0xffffffffu, v, src);
            if (act && lane == lead && ((peers >> src) & 1u)) v = AT::comb(v, ov);
          }
          if (follower) act = false;
          c = __popc(peers);
        }
        val[e] = v;
        go[e] = act && !(use_cache && cache_update(off[e], v, c));
        if constexpr (OP != kProd || PAIR) {
          if (go[e]) global_update(off[e], v, c);
        } else if constexpr (CNT) {
          if (go[e]) atomicAdd(cnt + off[e], c);  // the product itself is batched below
        }
      }
      if (probing) {
        agg = dups >= 4;
        probing = false;
      }
      if constexpr (OP == kProd && !PAIR) {
        __syncwarp();  // issue the batch from a converged warp
        A old[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (go[e]) old[e] = *reinterpret_cast<volatile A*>(acc + off[e]);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (go[e]) {
            bool ok;
            old[e] = cas_mul(acc + off[e], old[e], val[e], ok);
            go[e] = !ok;
          }
#pragma unroll
        for (int e = 0; e < 4; ++e)
          while (go[e]) {
            bool ok;
            old[e] = cas_mul(acc + off[e], old[e], val[e], ok);
            go[e] = !ok;
          }
      }
    };
    Quad qa, qb;
    int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t q0 = q - lane;  // the warp's first quad: loop bounds are warp-uniform
    load_quad(q, qa);
    for (int64_t w = q0; w < nq; w += 2 * stride, q += 2 * stride) {
      load_quad(q + stride, qb);
      do_quad(qa, q < nq);
      if (w + stride >= nq) break;
      load_quad(q + 2 * stride, qa);
      do_quad(qb, q + stride < nq);
    }
    for (int64_t p = nq * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n; p += stride) {
      const int64_t iv = (int64_t)index[p];
      if (iv < 0 || iv >= g.out_dim) { ++bad; continue; }
      update(iv * g.ostr[0], AT::from(src[p]));
    }
  } else {
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n; p += stride) {
      int64_t c[4] = {0, 0, 0, 0};
      int64_t rem = p;
#pragma unroll
      for (int d = NDIM - 1; d >= 0; --d) {
        c[d] = rem % g.shape[d];
        rem /= g.shape[d];
      }
      int64_t io = 0, so = 0, oo = 0;
#pragma unroll
      for (int d = 0; d < NDIM; ++d) {
        io += c[d] * g.istr[d];
        so += c[d] * g.sstr[d];
        if (d != g.dim) oo += c[d] * g.ostr[d];
      }
      const int64_t iv = (int64_t)index[io];
      if (iv < 0 || iv >= g.out_dim) { ++bad; continue; }
      update(oo + iv * g.ostr[g.dim], AT::from(src[so]));
    }
  }

  if (bad && err) atomicAdd(err, bad);
  if (use_cache) {
    __syncthreads();
    for (int j = threadIdx.x; j < kSlots; j += blockDim.x) {
      const uint32_t t = s_tag[j];
      if (t != kEmpty) {
        if constexpr (PAIR) {
          red_pair(reinterpret_cast<float*>(acc) + 2 * (int64_t)t, (float)s_val[j], (float)s_cnt[j]);
        } else {
          AT::op(acc + t, s_val[j]);
          if (CNT) atomicAdd(cnt + t, s_cnt[j]);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// init / finalize over the output (out may be strided: walk its logical shape)
// ---------------------------------------------------------------------------
struct OutGeo {
  int64_t shape[4];
  int64_t str[4];
  int ndim;
  int64_t numel;
};

__device__ __forceinline__ int64_t out_offset(const OutGeo& o, int64_t i) {
  int64_t off = 0;
  for (int d = o.ndim - 1; d >= 0; --d) {
    off += (i % o.shape[d]) * o.str[d];
    i /= o.shape[d];
  }
  return off;
}

template <typename T, int OP, bool KEYS, bool PAIR>
__global__ void scatter_init_kernel(const T* __restrict__ out, typename Acc<T, OP, KEYS>::A* acc,
                                    int32_t* cnt, OutGeo o, bool include_self) {
  using AT = Acc<T, OP, KEYS>;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < o.numel;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t off = out_offset(o, i);
    // the accumulator is indexed by the out offset (same strides as out)
    if constexpr (PAIR) {
      reinterpret_cast<float2*>(acc)[off] =
          make_float2(include_self ? (float)AT::from(out[off]) : 0.f, 0.f);
    } else {
      acc[off] = include_self ? AT::from(out[off]) : AT::identity();
      if (cnt) cnt[off] = 0;
    }
  }
}

template <typename T> __device__ __forceinline__ T from_acc(float a) { return from_f<T>(a); }
template <> __device__ __forceinline__ int32_t from_acc<int32_t>(float a) { return (int32_t)a; }

template <typename T, int OP, bool KEYS, bool PAIR>
__global__ void scatter_finalize_kernel(T* __restrict__ out,
                                        const typename Acc<T, OP, KEYS>::A* __restrict__ acc,
                                        const int32_t* __restrict__ cnt, OutGeo o,
                                        bool include_self, bool acc_is_out) {
  using AT = Acc<T, OP, KEYS>;
  using A = typename AT::A;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < o.numel;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t off = out_offset(o, i);
    if constexpr (KEYS) {
      const uint32_t k = (uint32_t)acc[off];
      if (!include_self && k == (uint32_t)AT::identity()) continue;  // never reached
      out[off] = from_f<T>(funkey(k));
      continue;
    } else {
    A a;
    int32_t c;
    if constexpr (PAIR) {
      const float2 pr = reinterpret_cast<const float2*>(acc)[off];
      a = (A)pr.x;
      c = (int32_t)pr.y;
    } else {
      c = cnt ? cnt[off] : 1;
      a = acc_is_out ? (A)0 : acc[off];
    }
    if (!include_self && c == 0) continue;  // never reached: keeps self
    if (OP == kMean) {
      const int32_t den = include_self ? c + 1 : c;
      if constexpr (std::is_same<A, float>::value) {
        const float s = acc_is_out ? tof<T>(out[off]) : a;
        out[off] = from_f<T>(s / (float)den);
      } else {
        const A s = acc_is_out ? (A)reinterpret_cast<const A*>(out)[off] : a;
        A q = s / (A)den;
        if ((s % (A)den != 0) && ((s < 0) != (den < 0))) q -= 1;  // floor division
        reinterpret_cast<A*>(out)[off] = q;
      }
    } else if (!acc_is_out) {
      if constexpr (std::is_same<A, float>::value) out[off] = from_f<T>(a);
      else reinterpret_cast<A*>(out)[off] = a;
    }
    }
  }
}

// ---------------------------------------------------------------------------
// destination-binned path (1-D contiguous updates, 4-byte accumulators, many
// updates): instead of one L2 atomic per update, three passes
//   count: updates per output slice of kSliceCells cells (shared histogram),
//   bin:   (slice << 13 | cell, value) pairs written slice-contiguously (each
//          CTA sorts a batch of 4096 updates by slice in shared memory and
//          appends every slice's run at a cursor reserved with one atomic),
//   reduce: segments of <= kSeg pairs of one slice applied to a dense
//          shared-memory copy of the slice, then merged into the accumulator
//          with one global operation per touched cell.
// The accumulator layout, init and finalize are those of the atomic path.
// Costs ~2.8x the algorithmic bytes, but at HBM rate instead of the L2's
// atomic request rate, and products need no global compare-and-swap loop per
// update.
// ---------------------------------------------------------------------------
constexpr int kSliceLog = 13;
constexpr int kSliceCells = 1 << kSliceLog;
constexpr int kMaxSlices = 1024;
constexpr int kBinBatch = 4096;  // updates per CTA step of the bin pass (512 threads x 8)
constexpr int64_t kSeg = 65536;   // pairs per reduce segment
constexpr int64_t kBinMinUpdates = (int64_t)1 << 20;
constexpr size_t kBinHeaderBytes = 12288;  // totals, cursors, work counter

// 4-byte accumulator <-> the 32 bits of a pair entry (bit copies, not value casts)
template <typename A> __device__ __forceinline__ uint32_t acc_bits(A v) {
  static_assert(sizeof(A) == 4, "4-byte accumulators");
  uint32_t u;
  memcpy(&u, &v, 4);
  return u;
}
template <typename A> __device__ __forceinline__ A acc_from_bits(uint32_t u) {
  A v;
  memcpy(&v, &u, 4);
  return v;
}

// Exclusive scan of v[0..n) (n <= 1024) into out[0..n] (out[n] = total) by a
// 512-thread block; v and out may alias.
__device__ __forceinline__ void block_scan_1024(const uint32_t* v, uint32_t* out, int n,
                                                uint32_t* warp_tot) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const uint32_t a = (2 * t < n) ? v[2 * t] : 0u, b = (2 * t + 1 < n) ? v[2 * t + 1] : 0u;
  uint32_t x = a + b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[w] = x;
  __syncthreads();
  if (w == 0) {
    uint32_t z = lane < 16 ? warp_tot[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, z, o);
      if (lane >= o) z += y;
    }
    if (lane < 16) warp_tot[lane] = z;  // inclusive warp totals
  }
  __syncthreads();
  const uint32_t before = (w > 0 ? warp_tot[w - 1] : 0u) + x - (a + b);
  if (2 * t < n) out[2 * t] = before;
  if (2 * t + 1 < n) out[2 * t + 1] = before + a;
  if (t == 0) out[n] = warp_tot[15];
  __syncthreads();
}

template <typename I>
__global__ void __launch_bounds__(512)
bin_count_kernel(const I* __restrict__ index, int64_t n, int64_t out_dim, int64_t ostr, int ns,
                 uint32_t* __restrict__ tot) {
  __shared__ uint32_t h[kMaxSlices];
  for (int i = threadIdx.x; i < ns; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
#pragma unroll 4
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n; p += stride) {
    const int64_t iv = (int64_t)index[p];
    if (iv >= 0 && iv < out_dim) atomicAdd(&h[(iv * ostr) >> kSliceLog], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < ns; i += blockDim.x)
    if (h[i]) atomicAdd(&tot[i], h[i]);
}

template <typename T, typename I, int OP, bool KEYS>
__global__ void __launch_bounds__(512)
bin_pairs_kernel(const T* __restrict__ src, const I* __restrict__ index, int64_t n,
                 int64_t out_dim, int64_t ostr, int ns, const uint32_t* __restrict__ tot,
                 uint32_t* __restrict__ cursor, uint2* __restrict__ pairs,
                 int32_t* __restrict__ err) {
  using AT = Acc<T, OP, KEYS>;
  using A = typename AT::A;
  static_assert(sizeof(A) == 4, "4-byte accumulators");
  __shared__ uint32_t s_start[kMaxSlices + 1];  // first pair of each slice
  __shared__ uint32_t s_cnt[kMaxSlices + 1];    // this batch: updates per slice, then offsets
  __shared__ uint32_t s_base[kMaxSlices];       // this batch: the slice run's place in the slice
  __shared__ uint32_t s_wt[16];
  __shared__ uint2 s_buf[kBinBatch];
  const int t = threadIdx.x;
  block_scan_1024(tot, s_start, ns, s_wt);
  int32_t bad = 0;
  // this thread's 8 updates of a batch, loaded one batch ahead
  int64_t niv[8];
  T nsv[8];
  uint32_t nin = 0;  // bit u: update u exists (not past the end)
  auto load_batch = [&](int64_t b0) {
    nin = 0;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t p = b0 + t + 512 * u;
      if (p < n) {
        niv[u] = (int64_t)index[p];
        nsv[u] = src[p];
        nin |= 1u << u;
      }
    }
  };
  const int64_t bstep = (int64_t)gridDim.x * kBinBatch;
  load_batch((int64_t)blockIdx.x * kBinBatch);
  for (int64_t b0 = (int64_t)blockIdx.x * kBinBatch; b0 < n; b0 += bstep) {
    for (int i = t; i < ns; i += 512) s_cnt[i] = 0;
    int64_t iv_[8];
    T sv_[8];
    const uint32_t in_ = nin;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      iv_[u] = niv[u];
      sv_[u] = nsv[u];
    }
    load_batch(b0 + bstep);
    __syncthreads();
    uint32_t w0[8], w1[8], lpos[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      w0[u] = 0xffffffffu;
      if (!((in_ >> u) & 1u)) continue;
      const int64_t iv = iv_[u];
      if (iv >= 0 && iv < out_dim) {
        const int64_t off = iv * ostr;
        w0[u] = (uint32_t)off;  // (slice << 13) | cell: off < ns * 8192 <= 2^23
        w1[u] = acc_bits<A>(AT::from(sv_[u]));
        lpos[u] = atomicAdd(&s_cnt[off >> kSliceLog], 1u);
      } else {
        ++bad;
      }
    }
    __syncthreads();
    // reserve each slice's run, then turn the counts into batch offsets
    for (int i = t; i < ns; i += 512)
      if (s_cnt[i]) s_base[i] = atomicAdd(&cursor[i], s_cnt[i]);
    __syncthreads();
    block_scan_1024(s_cnt, s_cnt, ns, s_wt);
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (w0[u] != 0xffffffffu) s_buf[s_cnt[w0[u] >> kSliceLog] + lpos[u]] = make_uint2(w0[u], w1[u]);
    __syncthreads();
    const uint32_t m = s_cnt[ns];
    for (uint32_t i = t; i < m; i += 512) {
      const uint2 e = s_buf[i];
      const uint32_t sl = e.x >> kSliceLog;
      pairs[(int64_t)s_start[sl] + s_base[sl] + (i - s_cnt[sl])] = e;
    }
    __syncthreads();
  }
  if (bad && err) atomicAdd(err, bad);
}

template <typename T, int OP, bool KEYS, bool CNT, bool PAIR>
__global__ void __launch_bounds__(512)
bin_reduce_kernel(const uint2* __restrict__ pairs, const uint32_t* __restrict__ tot, int ns,
                  int64_t span, uint32_t* __restrict__ next,
                  typename Acc<T, OP, KEYS>::A* __restrict__ acc, int32_t* __restrict__ cnt) {
  using AT = Acc<T, OP, KEYS>;
  using A = typename AT::A;
  constexpr bool kCnt = CNT || PAIR;
  extern __shared__ __align__(16) uint8_t bin_smem[];
  A* s_acc = reinterpret_cast<A*>(bin_smem);
  int32_t* s_c = reinterpret_cast<int32_t*>(bin_smem + kSliceCells * sizeof(A));
  __shared__ uint32_t s_start[kMaxSlices + 1];
  __shared__ uint32_t s_seg[kMaxSlices + 1];
  __shared__ uint32_t s_wt[16];
  __shared__ uint32_t s_w;
  const int t = threadIdx.x;
  block_scan_1024(tot, s_start, ns, s_wt);
  for (int i = t; i < ns; i += 512) s_seg[i] = (uint32_t)((tot[i] + kSeg - 1) / kSeg);
  __syncthreads();
  block_scan_1024(s_seg, s_seg, ns, s_wt);
  const uint32_t nseg = s_seg[ns];
  const A ident = AT::identity();
  for (;;) {
    if (t == 0) s_w = atomicAdd(next, 1u);
    __syncthreads();
    const uint32_t w = s_w;
    if (w >= nseg) break;
    // the slice holding segment w (s_seg is nondecreasing)
    int lo = 0, hi = ns - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_seg[mid] <= w) lo = mid;
      else hi = mid - 1;
    }
    const int sl = lo;
    const int64_t e0 = (int64_t)s_start[sl] + (int64_t)(w - s_seg[sl]) * kSeg;
    const int64_t e1 = min(e0 + kSeg, (int64_t)s_start[sl] + (int64_t)tot[sl]);
    for (int c = t; c < kSliceCells; c += 512) {
      s_acc[c] = ident;
      if (kCnt) s_c[c] = 0;
    }
    __syncthreads();
    int64_t e = e0 + t;
    for (; e + 3 * 512 < e1; e += 4 * 512) {  // four pairs in flight per thread
      uint2 pr[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) pr[u] = pairs[e + u * 512];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t c = pr[u].x & (kSliceCells - 1);
        AT::op(&s_acc[c], acc_from_bits<A>(pr[u].y));
        if (kCnt) atomicAdd(&s_c[c], 1);
      }
    }
    for (; e < e1; e += 512) {
      const uint2 pr = pairs[e];
      const uint32_t c = pr.x & (kSliceCells - 1);
      AT::op(&s_acc[c], acc_from_bits<A>(pr.y));
      if (kCnt) atomicAdd(&s_c[c], 1);
    }
    __syncthreads();
    const int64_t base = (int64_t)sl << kSliceLog;
    for (int c = t; c < kSliceCells && base + c < span; c += 512) {
      const A v = s_acc[c];
      const int64_t off = base + c;
      if constexpr (kCnt) {
        const int32_t k = s_c[c];
        if (k == 0) continue;
        if constexpr (PAIR) {
          red_pair(reinterpret_cast<float*>(acc) + 2 * off, (float)v, (float)k);
        } else {
          AT::op(acc + off, v);
          atomicAdd(cnt + off, k);
        }
      } else {
        if (v == ident) continue;  // an untouched cell, or a no-op merge
        AT::op(acc + off, v);
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// planning + dispatch
// ---------------------------------------------------------------------------
inline bool is_float(int dt) { return dt == FO_F32 || dt == FO_F16 || dt == FO_BF16; }
inline size_t round256(size_t b) { return (b + 255) & ~(size_t)255; }

struct Plan {
  bool keys;     // float amax/amin via uint32 keys in scratch
  bool scratch;  // accumulator in scratch (else directly in out)
  bool counts;   // int32 counts in scratch
  bool pair;     // interleaved float (sum, count) pairs in scratch (set per call)
  size_t acc_bytes, cnt_bytes;
  bool binned;   // destination-binned update pass (set per call)
  size_t bin_bytes;
};

// Workspace beyond the plan for the destination-binned path: slice totals,
// cursors and the work counter (a 12 KiB block: 4 KiB, 4 KiB, 4 bytes), then
// n (cell, value) pairs; 0 when the path does not apply.
// Used for products: their atomic path is a load and a compare-and-swap loop
// per update (0.41 ms uniform / 0.87 ms Zipf at 2^24 updates into 2^20 cells),
// the binned passes take 0.26 / 0.60 ms.  For sum, mean, amax and amin the
// L2's atomic units stay faster (0.12-0.19 ms against 0.24-0.46 ms binned).
inline size_t binned_bytes(int reduce, int dtype, int64_t span, int64_t n) {
  const bool four = dtype == FO_F32 || dtype == FO_F16 || dtype == FO_BF16 || dtype == FO_I32;
  if (reduce != FO_PROD || !four || n < kBinMinUpdates || span <= 0 ||
      span > (int64_t)kMaxSlices * kSliceCells)
    return 0;
  return kBinHeaderBytes + round256((size_t)n * 8);
}

// Float sum without self and float mean may use (sum, count) pairs; the
// workspace covers both that layout and separate float sums + int32 counts.
inline bool pair_capable(int reduce, bool include_self, int dtype) {
  return is_float(dtype) && (reduce == FO_MEAN || (reduce == FO_SUM && !include_self));
}

Plan make_plan(int reduce, bool include_self, int dtype, int64_t span) {
  Plan p{};
  const bool f = is_float(dtype);
  const bool half = dtype == FO_F16 || dtype == FO_BF16;
  p.keys = f && (reduce == FO_AMAX || reduce == FO_AMIN);
  p.counts = (reduce == FO_MEAN) || (!include_self && !p.keys);
  p.scratch = p.keys || !include_self || half || pair_capable(reduce, include_self, dtype);
  size_t asz = p.keys ? 4 : (f ? 4 : dtype_size(dtype));
  p.acc_bytes = p.scratch ? round256((size_t)span * asz) : 0;
  p.cnt_bytes = p.counts ? round256((size_t)span * 4) : 0;
  return p;
}

// Per-call choice: pairs when every count fits a float exactly (<= 2^24 updates).
inline void choose_pairs(Plan& p, int reduce, bool include_self, int dtype, int64_t n) {
  p.pair = pair_capable(reduce, include_self, dtype) && n <= ((int64_t)1 << 24);
}

// number of elements an out-offset-indexed array must cover
int64_t out_span(const int64_t* shape, const int64_t* str, int ndim) {
  int64_t m = 0;
  for (int d = 0; d < ndim; ++d) {
    if (shape[d] == 0) return 0;
    m += (shape[d] - 1) * str[d];
  }
  return m + 1;
}

template <typename T, typename I, int OP, bool KEYS>
int run(void* out, const void* src, const void* index, const Geo& g, const OutGeo& og,
        int64_t n, bool include_self, const Plan& pl, void* ws, int32_t* err, cudaStream_t st) {
  using AT = Acc<T, OP, KEYS>;
  using A = typename AT::A;
  A* acc = pl.scratch ? reinterpret_cast<A*>(ws) : reinterpret_cast<A*>(out);
  int32_t* cnt = (pl.counts && !pl.pair) ? reinterpret_cast<int32_t*>((char*)ws + pl.acc_bytes)
                                         : nullptr;
  constexpr bool kPairable = std::is_same<A, float>::value && !KEYS && (OP == kSum || OP == kMean);
  const int sms = num_sms();
  if (pl.scratch) {
    int64_t gi = (og.numel + 255) / 256;
    if (gi > sms * 8) gi = sms * 8;
    if (gi < 1) gi = 1;
    if (kPairable && pl.pair)
      scatter_init_kernel<T, OP, KEYS, kPairable><<<(unsigned)gi, 256, 0, st>>>(
          (const T*)out, acc, nullptr, og, include_self);
    else
      scatter_init_kernel<T, OP, KEYS, false><<<(unsigned)gi, 256, 0, st>>>((const T*)out, acc, cnt,
                                                                           og, include_self);
    if (int rc = check_launch("scatter_init_kernel")) return rc;
  } else if (cnt) {
    cudaMemsetAsync(cnt, 0, pl.cnt_bytes, st);
  }
  if (n > 0 && pl.binned) {
    // destination-binned pass: 1-D contiguous index and src (checked by the caller)
    const int64_t span = out_span(og.shape, og.str, og.ndim);
    const int ns = (int)((span + kSliceCells - 1) / kSliceCells);
    char* bw = reinterpret_cast<char*>(ws) + pl.acc_bytes + pl.cnt_bytes;
    uint32_t* tot = reinterpret_cast<uint32_t*>(bw);
    uint32_t* cursor = tot + kMaxSlices;
    uint32_t* next = cursor + kMaxSlices;
    uint2* pairs = reinterpret_cast<uint2*>(bw + kBinHeaderBytes);
    if constexpr (sizeof(A) == 4) {
      if (cudaMemsetAsync(bw, 0, kBinHeaderBytes, st) != cudaSuccess) {
        set_error("scatter_reduce: cudaMemsetAsync failed");
        return FO_ECUDA;
      }
      bin_count_kernel<I><<<sms * 4, 512, 0, st>>>((const I*)index, n, g.out_dim, g.ostr[0], ns,
                                                   tot);
      if (int rc = check_launch("bin_count_kernel")) return rc;
      int64_t gb = (n + kBinBatch - 1) / kBinBatch;
      if (gb > (int64_t)sms * 4) gb = (int64_t)sms * 4;
      bin_pairs_kernel<T, I, OP, KEYS><<<(unsigned)gb, 512, 0, st>>>(
          (const T*)src, (const I*)index, n, g.out_dim, g.ostr[0], ns, tot, cursor, pairs, err);
      if (int rc = check_launch("bin_pairs_kernel")) return rc;
      const bool with_cnt = (cnt != nullptr) || (kPairable && pl.pair);
      const int smem = (int)(kSliceCells * sizeof(A)) + (with_cnt ? kSliceCells * 4 : 0);
#define FO_BIN_REDUCE(C, P)                                                                    \
  {                                                                                            \
    auto rk = bin_reduce_kernel<T, OP, KEYS, C, P>;                                            \
    if (cudaFuncSetAttribute(rk, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=         \
        cudaSuccess) {                                                                         \
      set_error("scatter_reduce: cannot reserve %d bytes of shared memory", smem);            \
      return FO_ECUDA;                                                                         \
    }                                                                                          \
    rk<<<sms * 3, 512, smem, st>>>(pairs, tot, ns, span, next, acc, cnt);                      \
  }
      if (kPairable && pl.pair) FO_BIN_REDUCE(false, kPairable)
      else if (cnt) FO_BIN_REDUCE(true, false)
      else FO_BIN_REDUCE(false, false)
#undef FO_BIN_REDUCE
      if (int rc = check_launch("bin_reduce_kernel")) return rc;
    }
  } else if (n > 0) {
    const int64_t span = out_span(og.shape, og.str, og.ndim);
    const bool use_cache = span < (int64_t)0xffffffffLL;
    int64_t grid = (n + (int64_t)kThreads * 16 - 1) / ((int64_t)kThreads * 16);
    if (grid > (int64_t)sms * 2) grid = (int64_t)sms * 2;
    if (grid < 1) grid = 1;
    const bool vec = g.ndim == 1 && sizeof(I) == 8 && g.istr[0] == 1 && g.sstr[0] == 1 &&
                     aligned16(index) && aligned16(src);
#define FO_LAUNCH(ND, V)                                                                       \
  scatter_kernel<T, I, OP, KEYS, true, false, ND, V><<<(unsigned)grid, kThreads, 0, st>>>(     \
      (const T*)src, (const I*)index, acc, cnt, n, g, err, use_cache)
#define FO_LAUNCH_NC(ND, V)                                                                    \
  scatter_kernel<T, I, OP, KEYS, false, false, ND, V><<<(unsigned)grid, kThreads, 0, st>>>(    \
      (const T*)src, (const I*)index, acc, nullptr, n, g, err, use_cache)
#define FO_LAUNCH_PAIR(ND, V)                                                                  \
  scatter_kernel<T, I, OP, KEYS, false, kPairable, ND, V><<<(unsigned)grid, kThreads, 0, st>>>( \
      (const T*)src, (const I*)index, acc, nullptr, n, g, err, use_cache)
    if (kPairable && pl.pair) {
      if (vec) FO_LAUNCH_PAIR(1, (sizeof(I) == 8));
      else if (g.ndim == 1) FO_LAUNCH_PAIR(1, false);
      else if (g.ndim == 2) FO_LAUNCH_PAIR(2, false);
      else if (g.ndim == 3) FO_LAUNCH_PAIR(3, false);
      else FO_LAUNCH_PAIR(4, false);
    } else if (cnt) {
      if (vec) FO_LAUNCH(1, (sizeof(I) == 8));
      else if (g.ndim == 1) FO_LAUNCH(1, false);
      else if (g.ndim == 2) FO_LAUNCH(2, false);
      else if (g.ndim == 3) FO_LAUNCH(3, false);
      else FO_LAUNCH(4, false);
    } else {
      if (vec) FO_LAUNCH_NC(1, (sizeof(I) == 8));
      else if (g.ndim == 1) FO_LAUNCH_NC(1, false);
      else if (g.ndim == 2) FO_LAUNCH_NC(2, false);
      else if (g.ndim == 3) FO_LAUNCH_NC(3, false);
      else FO_LAUNCH_NC(4, false);
    }
#undef FO_LAUNCH
#undef FO_LAUNCH_NC
#undef FO_LAUNCH_PAIR
    if (int rc = check_launch("scatter_kernel")) return rc;
  }
  if (pl.scratch || OP == kMean) {
    int64_t gf = (og.numel + 255) / 256;
    if (gf > sms * 8) gf = sms * 8;
    if (gf < 1) gf = 1;
    if (kPairable && pl.pair)
      scatter_finalize_kernel<T, OP, KEYS, kPairable><<<(unsigned)gf, 256, 0, st>>>(
          (T*)out, acc, nullptr, og, include_self, false);
    else
      scatter_finalize_kernel<T, OP, KEYS, false><<<(unsigned)gf, 256, 0, st>>>(
          (T*)out, acc, cnt, og, include_self, !pl.scratch);
    if (int rc = check_launch("scatter_finalize_kernel")) return rc;
  }
  return FO_OK;
}

template <typename T, typename I>
int dispatch_op(int reduce, void* out, const void* src, const void* index, const Geo& g,
                const OutGeo& og, int64_t n, bool inc, const Plan& pl, void* ws, int32_t* err,
                cudaStream_t st) {
  constexpr bool F = std::is_same<T, float>::value || std::is_same<T, __half>::value ||
                     std::is_same<T, __nv_bfloat16>::value;
  switch (reduce) {
    case FO_SUM: return run<T, I, kSum, false>(out, src, index, g, og, n, inc, pl, ws, err, st);
    case FO_PROD: return run<T, I, kProd, false>(out, src, index, g, og, n, inc, pl, ws, err, st);
    case FO_MEAN: return run<T, I, kMean, false>(out, src, index, g, og, n, inc, pl, ws, err, st);
    case FO_AMAX: return run<T, I, kAmax, F>(out, src, index, g, og, n, inc, pl, ws, err, st);
    case FO_AMIN: return run<T, I, kAmin, F>(out, src, index, g, og, n, inc, pl, ws, err, st);
  }
  set_error("scatter_reduce: Unsupported reduce code %d", reduce);
  return FO_EINVAL;
}

template <typename I>
int dispatch_dtype(int dtype, int reduce, void* out, const void* src, const void* index,
                   const Geo& g, const OutGeo& og, int64_t n, bool inc, const Plan& pl, void* ws,
                   int32_t* err, cudaStream_t st) {
  switch (dtype) {
    case FO_F32: return dispatch_op<float, I>(reduce, out, src, index, g, og, n, inc, pl, ws, err, st);
    case FO_F16: return dispatch_op<__half, I>(reduce, out, src, index, g, og, n, inc, pl, ws, err, st);
    case FO_BF16:
      return dispatch_op<__nv_bfloat16, I>(reduce, out, src, index, g, og, n, inc, pl, ws, err, st);
    case FO_I32: return dispatch_op<int32_t, I>(reduce, out, src, index, g, og, n, inc, pl, ws, err, st);
    case FO_I64: return dispatch_op<int64_t, I>(reduce, out, src, index, g, og, n, inc, pl, ws, err, st);
  }
  set_error("scatter_reduce: unsupported dtype code %d", dtype);
  return FO_EDTYPE;
}

}  // namespace
}  // namespace fo

using namespace fo;

extern "C" int fo_scatter_reduce_workspace_bytes(int64_t out_numel, int reduce, int include_self,
                                                 int dtype, int64_t* bytes) {
  clear_error();
  FO_CHECK_ARG(bytes && out_numel >= 0, "fo_scatter_reduce_workspace_bytes: bad argument");
  FO_CHECK_ARG(reduce >= FO_SUM && reduce <= FO_AMIN, "Unsupported reduce code %d", reduce);
  const Plan p = make_plan(reduce, include_self != 0, dtype, out_numel);
  *bytes = (int64_t)(p.acc_bytes + p.cnt_bytes);
  return FO_OK;
}

namespace fo {
namespace {
inline bool known_dtype(int dt) {
  return dt == FO_F32 || dt == FO_F16 || dt == FO_BF16 || dt == FO_I32 || dt == FO_I64;
}

// Argument checks shared by both scatter entry points (same status codes and
// messages), and the kernel geometry of the call.
int prepare_scatter(const void* out, const void* src, const void* index, int ndim,
                    const int64_t* index_shape, const int64_t* index_strides,
                    const int64_t* src_strides, const int64_t* out_shape,
                    const int64_t* out_strides, int dim, int reduce, int dtype, int index_dtype,
                    Geo& g, OutGeo& og, int64_t& n) {
  FO_CHECK_ARG(ndim >= 1 && ndim <= 4, "scatter_reduce supports 1-4-D tensors, got %dD", ndim);
  FO_CHECK_ARG(dim >= 0 && dim < ndim, "scatter_reduce: dim %d out of range", dim);
  FO_CHECK_ARG(reduce >= FO_SUM && reduce <= FO_AMIN, "Unsupported reduce code %d", reduce);
  FO_CHECK_ARG(index_dtype == FO_I64 || index_dtype == FO_I32,
               "scatter_reduce: index must be int64 or int32");
  FO_CHECK_ARG(index_shape && index_strides && src_strides && out_shape && out_strides,
               "scatter_reduce: null shape/stride array");
  if (!known_dtype(dtype)) {
    set_error("scatter_reduce: unsupported dtype code %d", dtype);
    return FO_EDTYPE;
  }
  g = Geo{};
  og = OutGeo{};
  n = 1;
  og.numel = 1;
  for (int d = 0; d < 4; ++d) {
    g.shape[d] = d < ndim ? index_shape[d] : 1;
    g.istr[d] = d < ndim ? index_strides[d] : 0;
    g.sstr[d] = d < ndim ? src_strides[d] : 0;
    g.ostr[d] = d < ndim ? out_strides[d] : 0;
    og.shape[d] = d < ndim ? out_shape[d] : 1;
    og.str[d] = d < ndim ? out_strides[d] : 0;
    FO_CHECK_ARG(g.shape[d] >= 0 && og.shape[d] >= 0, "scatter_reduce: negative shape");
    FO_CHECK_ARG(g.istr[d] >= 0 && g.sstr[d] >= 0 && og.str[d] >= 0,
                 "scatter_reduce: negative stride");
    n *= g.shape[d];
    og.numel *= og.shape[d];
  }
  for (int d = 0; d < ndim; ++d)
    FO_CHECK_ARG(d == dim || index_shape[d] <= out_shape[d],
                 "scatter_reduce: index size %lld > self size %lld at dim %d",
                 (long long)index_shape[d], (long long)out_shape[d], d);
  g.out_dim = out_shape[dim];
  g.dim = dim;
  g.ndim = ndim;
  og.ndim = ndim;
  if (og.numel == 0) return FO_OK;
  FO_CHECK_ARG(out && (n == 0 || (src && index)), "scatter_reduce: null pointer");
  return FO_OK;
}
}  // namespace
}  // namespace fo

extern "C" int fo_scatter_reduce_binned_bytes(int64_t out_span, int64_t n, int reduce, int dtype,
                                              int64_t* bytes) {
  clear_error();
  FO_CHECK_ARG(bytes && out_span >= 0 && n >= 0, "fo_scatter_reduce_binned_bytes: bad argument");
  *bytes = (int64_t)binned_bytes(reduce, dtype, out_span, n);
  return FO_OK;
}

extern "C" int fo_scatter_reduce(void* out, const void* src, const void* index, int ndim,
                                 const int64_t* index_shape, const int64_t* index_strides,
                                 const int64_t* src_strides, const int64_t* out_shape,
                                 const int64_t* out_strides, int dim, int reduce,
                                 int include_self, int dtype, int index_dtype, void* workspace,
                                 int64_t ws_bytes, int32_t* err_count, void* stream) {
  clear_error();
  Geo g;
  OutGeo og;
  int64_t n = 0;
  if (int rc = prepare_scatter(out, src, index, ndim, index_shape, index_strides, src_strides,
                               out_shape, out_strides, dim, reduce, dtype, index_dtype, g, og, n))
    return rc;
  if (og.numel == 0) return FO_OK;
  const int64_t span = out_span(og.shape, og.str, ndim);
  Plan pl = make_plan(reduce, include_self != 0, dtype, span);
  choose_pairs(pl, reduce, include_self != 0, dtype, n);
  if ((int64_t)(pl.acc_bytes + pl.cnt_bytes) > 0 &&
      (!workspace || ws_bytes < (int64_t)(pl.acc_bytes + pl.cnt_bytes))) {
    set_error("scatter_reduce: workspace of %lld bytes required, got %lld",
              (long long)(pl.acc_bytes + pl.cnt_bytes), (long long)ws_bytes);
    return FO_EWORKSPACE;
  }
  // the destination-binned pass when it applies and the caller's workspace
  // holds its pairs (fo_scatter_reduce_binned_bytes); else per-update atomics
  pl.bin_bytes = binned_bytes(reduce, dtype, span, n);
  pl.binned = pl.bin_bytes > 0 && ndim == 1 && g.istr[0] == 1 && g.sstr[0] == 1 && workspace &&
              aligned16(workspace) &&
              ws_bytes >= (int64_t)(pl.acc_bytes + pl.cnt_bytes + pl.bin_bytes);
  cudaStream_t st = as_stream(stream);
  if (index_dtype == FO_I64)
    return dispatch_dtype<int64_t>(dtype, reduce, out, src, index, g, og, n, include_self != 0, pl,
                                   workspace, err_count, st);
  return dispatch_dtype<int32_t>(dtype, reduce, out, src, index, g, og, n, include_self != 0, pl,
                                 workspace, err_count, st);
}

// ---------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot allocate device memory at the moment they need a
// scatter: a host framework that owns the whole device heap (pre-reserved
// memory pools that forbid any other allocation), a foreign-function caller
// (cgo, JNI, a plugin host) that has no handle to the program's allocator, or
// code that must not pay the implicit device synchronisation a cudaMalloc can
// trigger.  For them the scratch (accumulator + counts) lives in one
// file-scope device array, reserved when the library is loaded on a device and
// held by every device that loads it until the process exits.
// ---------------------------------------------------------------------------
#include <mutex>

namespace fo {
namespace {
// Accumulator + counts for an output whose memory span (1 + sum over dims of
// (size - 1) * stride, in elements) is at most 2^20, 8-byte accumulators
// included: 12 MiB per device.
constexpr size_t kNoAllocScratchBytes = (size_t)12 << 20;
__device__ __align__(256) unsigned char g_scatter_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {nullptr};

// Device address of g_scatter_scratch on the current device, looked up once per
// device with that device current (the symbol's name in host code is a
// host-side stand-in, not a device address).  The cached address belongs to the
// device's primary context: after cudaDeviceReset the library's device code is
// loaded again and the address may change, so the entry point must not be used
// after a device reset in the same process.
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("scatter_reduce_noalloc: no usable current device");
    return FO_ECUDA;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_scatter_scratch);
    if (e != cudaSuccess || !p) {
      set_error("scatter_reduce_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return FO_ECUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return FO_OK;
}
}  // namespace
}  // namespace fo

extern "C" int fo_scatter_reduce_noalloc(void* out, const void* src, const void* index, int ndim,
                                         const int64_t* index_shape,
                                         const int64_t* index_strides,
                                         const int64_t* src_strides, const int64_t* out_shape,
                                         const int64_t* out_strides, int dim, int reduce,
                                         int include_self, int dtype, int index_dtype,
                                         int32_t* err_count, void* stream) {
  clear_error();
  Geo g;
  OutGeo og;
  int64_t n = 0;
  if (int rc = prepare_scatter(out, src, index, ndim, index_shape, index_strides, src_strides,
                               out_shape, out_strides, dim, reduce, dtype, index_dtype, g, og, n))
    return rc;
  if (og.numel == 0) return FO_OK;
  const int64_t span = out_span(og.shape, og.str, ndim);
  const Plan pl = make_plan(reduce, include_self != 0, dtype, span);
  const size_t need = pl.acc_bytes + pl.cnt_bytes;
  if (need > kNoAllocScratchBytes) {
    set_error("scatter_reduce_noalloc: this call needs %zu bytes of scratch but the static "
              "scratch holds %zu (an output memory span of at most 2^20 elements); use "
              "fo_scatter_reduce with a caller-provided workspace", need, kNoAllocScratchBytes);
    return FO_EWORKSPACE;
  }
  void* ws = nullptr;
  if (need > 0) {
    if (int rc = scratch_address(&ws)) return rc;
  }
  // The scratch keeps the previous call's contents; the init pass of the
  // scatter clears every byte this call reads before it is used.
  return fo_scatter_reduce(out, src, index, ndim, index_shape, index_strides, src_strides,
                           out_shape, out_strides, dim, reduce, include_self, dtype, index_dtype,
                           ws, (int64_t)kNoAllocScratchBytes, err_count, stream);
}
