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
// Each pass histograms a digit of the elements whose higher digits equal the
// prefix selected so far and picks the bucket holding rank r.
//
// Rows of 1024 < N <= 2048 (4-byte types, 16-byte rows): producer warps stage
// the row's words and histogram their raw top 11 bits, consumer warps select
// (median_ws_kernel).  Rows of 256 < N <= 384 (4-byte types): one warp per row,
// the row in registers (median_warp_kernel).  Both read the histogram of raw
// top bits in value order, so no element is turned into a key before its bin
// is selected.
// Other rows of N <= 2048 (4-byte and smaller types): a group of RG = 1, 2 or 4 warps
// per row, 16 elements per thread in registers (16-byte vector loads when the
// row is 16-byte aligned; the next row is loaded while the current one is
// selected).  One pass over the top log2(512 RG) key bits, compaction of the
// selected bucket as 32-bit (key << digit bits | index) composites whose order
// is the stable sort order, and selection among them (rank counting for <= 32,
// radix passes otherwise).  NaN and infinite keys fall in the histogram's edge
// bins, so the NaN rule costs nothing per element unless those bins are used.
// Longer rows, int64 and the global median: one CTA per row, 11-bit digits,
// passes re-read the row (L2 hits for rows that fit in L2); after the last pass
// the key of the k-th element is known and the answer is found with ballots.
#include "common.cuh"
#include "tc05.cuh"

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
  static constexpr bool kHasNan = true;
  // NaN keys lie above the +inf key (0xff800000) or below the -inf key (0x007fffff)
  static __device__ __forceinline__ bool key_is_nan(uint32_t k) {
    return k > 0xff800000u || k < 0x007fffffu;
  }
  // +0.0 and -0.0 share one key; the stored element decides the sign of the value
  static __device__ __forceinline__ bool is_zero_key(uint32_t k) { return k == 0x80000000u; }
  static __device__ __forceinline__ float from_key(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k ^ 0x80000000u) : ~k);
  }
};
template <> struct KeyTraits<__half> {
  using K = uint32_t;
  static __device__ __forceinline__ K key(__half x) { return KeyTraits<float>::key(__half2float(x)); }
  static __device__ __forceinline__ bool isnan_(__half x) { return __hisnan(x); }
  static constexpr bool kHasNan = true;
  static __device__ __forceinline__ bool key_is_nan(uint32_t k) { return KeyTraits<float>::key_is_nan(k); }
  static __device__ __forceinline__ bool is_zero_key(uint32_t k) { return k == 0x80000000u; }
  static __device__ __forceinline__ __half from_key(uint32_t k) {
    return __float2half_rn(KeyTraits<float>::from_key(k));  // exact: the key came from a half
  }
};
template <> struct KeyTraits<__nv_bfloat16> {
  using K = uint32_t;
  static __device__ __forceinline__ K key(__nv_bfloat16 x) {
    return KeyTraits<float>::key(__bfloat162float(x));
  }
  static __device__ __forceinline__ bool isnan_(__nv_bfloat16 x) { return __hisnan(x); }
  static constexpr bool kHasNan = true;
  static __device__ __forceinline__ bool key_is_nan(uint32_t k) { return KeyTraits<float>::key_is_nan(k); }
  static __device__ __forceinline__ bool is_zero_key(uint32_t k) { return k == 0x80000000u; }
  static __device__ __forceinline__ __nv_bfloat16 from_key(uint32_t k) {
    return __float2bfloat16_rn(KeyTraits<float>::from_key(k));  // exact: the key came from a bf16
  }
};
template <> struct KeyTraits<int32_t> {
  using K = uint32_t;
  static __device__ __forceinline__ K key(int32_t x) { return (uint32_t)x ^ 0x80000000u; }
  static __device__ __forceinline__ bool isnan_(int32_t) { return false; }
  static constexpr bool kHasNan = false;
  static __device__ __forceinline__ bool key_is_nan(uint32_t) { return false; }
  static __device__ __forceinline__ bool is_zero_key(uint32_t) { return false; }
  static __device__ __forceinline__ int32_t from_key(uint32_t k) { return (int32_t)(k ^ 0x80000000u); }
};
template <> struct KeyTraits<int64_t> {
  using K = uint64_t;
  static __device__ __forceinline__ K key(int64_t x) { return (uint64_t)x ^ 0x8000000000000000ull; }
  static __device__ __forceinline__ bool isnan_(int64_t) { return false; }
  static __device__ __forceinline__ bool is_zero_key(uint64_t) { return false; }
  static __device__ __forceinline__ int64_t from_key(uint64_t k) {
    return (int64_t)(k ^ 0x8000000000000000ull);
  }
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
// row groups of RG warps (N <= 512 * RG): keys in registers, one radix pass,
// compaction of the selected bucket, selection on the compacted list
// ---------------------------------------------------------------------------
// Each thread holds 16 elements of the row.  Element e is held by warp w of the
// group, lane `lane`, slot (i, c):
//   e = ((i * RG + w) * 32 + lane) * VW + c          (16-byte vectors when VW > 1)
// The row group has kCap = 512 * RG slots; the first pass histograms the top
// kDig = log2(kCap) key bits into kCap bins (16 bins per thread).  The bucket's
// elements are compacted as 32-bit composites
//   (key << kDig) | e
// (the bucket's kDig key bits shift out, the index fills the freed bits), whose
// ascending order is the stable sort order of the bucket.
//
// The kernel is bound by the latency of its chain of shared-memory round trips
// and group barriers per row, so the chain is kept short: warp totals come from
// one redux, lane prefixes from bit-serial ballots (no shuffle chain), the
// compaction appends to per-warp lists with ballots (no atomic round trip), and
// the final selection reads all candidates with 16-byte loads.
template <int RG>
__device__ __forceinline__ void group_sync(int g) {
  if (RG == 1) __syncwarp();
  else asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(RG * 32) : "memory");
}

template <int RG>
struct RowGeom {
  static constexpr int kThreads = RG * 32;
  static constexpr int kCap = 16 * kThreads;
  static constexpr int kDig = RG == 1 ? 9 : (RG == 2 ? 10 : 11);
  static constexpr int kSh = 32 - kDig;
  static_assert((1 << kDig) == kCap, "one bin per slot");
};

// Bin b is stored at word hslot(b): bits 2-3 of b are XORed with bits 5-6, so
// the 16-byte chunks the scan reads (chunk j of thread t = bins 16t + 4j ..)
// land on distinct banks within every quarter warp (a 4-way conflict otherwise).
__device__ __forceinline__ uint32_t hslot(uint32_t b) { return b ^ ((b >> 3) & 0xcu); }

__device__ __forceinline__ uint32_t lanemask_le() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_le;" : "=r"(m));
  return m;
}
__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

template <int RG>
struct __align__(16) RowSmem {
  uint32_t hist[RowGeom<RG>::kCap];
  uint32_t list[RowGeom<RG>::kCap];  // RG per-warp regions of 512 composites
  uint32_t tmp[32];                  // candidates of the final selection
  uint32_t wsum[4];                  // per-warp totals (+ edge flags in bits 20+)
  uint32_t wcnt[4];                  // per-warp candidate counts
  uint32_t bucket, below, count, first_nan;
};

// Every thread owns 16 consecutive bins: it reads them, zeroes them for the
// next pass (no other thread reads them in this pass), and the group locates
// the bin holding rank r.  Returns to every thread that bin, the count below it
// and its count.  With `edge`, `special` reports a nonzero count in the first
// or last 4 bins (where NaN and infinite float keys fall); the flag rides in
// bits 20+ of the warp totals, above any count (counts <= 2048).
template <int RG>
__device__ __forceinline__ void row_find(RowSmem<RG>& S, int g, uint32_t r, bool edge,
                                         uint32_t& bin, uint32_t& below, uint32_t& cnt,
                                         bool& special) {
  constexpr int kTotBits = RowGeom<RG>::kDig + 1;  // a thread's total is <= kCap
  const int t = threadIdx.x & (RG * 32 - 1), lane = t & 31, w = t >> 5;
  uint4* hp = reinterpret_cast<uint4*>(S.hist + 16 * t);
  const int sw = (t >> 1) & 3;  // chunk j of this thread is stored at chunk j ^ sw
  uint4 h[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = hp[j ^ sw];
#pragma unroll
  for (int j = 0; j < 4; ++j) hp[j] = make_uint4(0, 0, 0, 0);
  const uint32_t c[16] = {h[0].x, h[0].y, h[0].z, h[0].w, h[1].x, h[1].y, h[1].z, h[1].w,
                          h[2].x, h[2].y, h[2].z, h[2].w, h[3].x, h[3].y, h[3].z, h[3].w};
  uint32_t tot = 0;
#pragma unroll
  for (int j = 0; j < 16; ++j) tot += c[j];
  uint32_t sp = 0;
  if (edge) {
    if (t == 0) sp = (c[0] | c[1] | c[2] | c[3]) != 0u;
    if (t == RG * 32 - 1) sp |= (c[12] | c[13] | c[14] | c[15]) != 0u;
  }
  const uint32_t wt = __reduce_add_sync(0xffffffffu, tot + (sp << 20));
  uint32_t off = 0, all = wt;
  int ow = 0;  // the warp whose bins hold rank r
  if (RG > 1) {
    if (lane == 0) S.wsum[w] = wt;
    group_sync<RG>(g);
    all = 0;
    uint32_t cum = 0;
#pragma unroll
    for (int q = 0; q < RG; ++q) {
      const uint32_t s = S.wsum[q];
      all += s;
      const uint32_t cq = s & 0xfffffu;
      if (ow == q && r >= cum + cq && q + 1 < RG) {
        cum += cq;
        ow = q + 1;
      }
    }
    off = cum;
  }
  special = (all >> 20) != 0u;
  if (w == ow) {
    // lane prefixes of the owner warp from one ballot per bit of the totals
    const uint32_t le = lanemask_le();
    uint32_t inc = 0;
#pragma unroll
    for (int b = 0; b < kTotBits; ++b)
      inc += (uint32_t)__popc(__ballot_sync(0xffffffffu, (tot >> b) & 1u) & le) << b;
    inc += off;
    const uint32_t exc = inc - tot;
    if (exc <= r && r < inc) {
      uint32_t acc = exc;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (r < acc + c[j]) {
          S.bucket = 16 * t + j;
          S.below = acc;
          S.count = c[j];
          break;
        }
        acc += c[j];
      }
    }
  }
  group_sync<RG>(g);
  bin = S.bucket;
  below = S.below;
  cnt = S.count;
}

// 4 CTAs per SM (64 registers) for rows that fill the group; the predicated
// variants need more registers.
template <typename T, int RG, int VW, bool FULL, int GPC>
__global__ void __launch_bounds__(GPC * RG * 32, FULL ? 4 : 3)
median_rows_kernel(const T* __restrict__ x, T* __restrict__ vals, int64_t* __restrict__ idxs,
                   int64_t M, int N) {
  using Tr = KeyTraits<T>;
  using G = RowGeom<RG>;
  static_assert(sizeof(typename Tr::K) == 4, "32-bit keys only");
  constexpr int NI = 16 / VW;
  constexpr int kSh = G::kSh, kDig = G::kDig;
  constexpr int kRegion = 512;  // list words per warp
  extern __shared__ __align__(16) uint8_t median_smem[];
  const int g = threadIdx.x / (RG * 32);
  const int t = threadIdx.x & (RG * 32 - 1);
  const int lane = t & 31, w = t >> 5;
  RowSmem<RG>& S = reinterpret_cast<RowSmem<RG>*>(median_smem)[g];
  const uint32_t k = (uint32_t)(N - 1) / 2;

#pragma unroll
  for (int j = 0; j < 4; ++j)
    reinterpret_cast<uint4*>(S.hist + 16 * t)[j] = make_uint4(0, 0, 0, 0);
  if (t == 0) S.first_nan = ~0u;
  group_sync<RG>(g);

  // The next row is loaded into registers while the current row is selected.
  constexpr int RV = VW > 1 ? NI : 1;
  constexpr int RS = VW > 1 ? 1 : 16;
  uint4 rv[RV];
  T rs[RS];
  auto load_row = [&](int64_t rrow) {
    if (rrow >= M) return;
    const T* xx = x + rrow * (int64_t)N;
    if constexpr (VW > 1) {
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        const int base = ((i * RG + w) * 32 + lane) * VW;
        rv[i] = (FULL || base < N) ? ld_global_stream_v4(xx + base) : make_uint4(0, 0, 0, 0);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int e = (i * RG + w) * 32 + lane;
        rs[i] = (FULL || e < N) ? xx[e] : T(0);
      }
    }
  };
  auto elem = [&](int i, int c) { return ((i * RG + w) * 32 + lane) * VW + c; };

  const int64_t row0 = (int64_t)blockIdx.x * GPC + g;
  const int64_t rstep = (int64_t)gridDim.x * GPC;
  load_row(row0);

  int fw = 0;  // the warp that finishes this row (rotates, so no warp lags)
  for (int64_t row = row0; row < M; row += rstep, fw = (fw + 1) & (RG - 1)) {
    uint32_t key[16];
#pragma unroll
    for (int i = 0; i < NI; ++i)
#pragma unroll
      for (int c = 0; c < VW; ++c) {
        if constexpr (VW > 1) key[i * VW + c] = Tr::key(reinterpret_cast<const T*>(&rv[i])[c]);
        else key[i] = Tr::key(rs[i]);
      }
    load_row(row + rstep);

    // ---- pass 0 over registers: top kDig bits
#pragma unroll
    for (int i = 0; i < NI; ++i)
#pragma unroll
      for (int c = 0; c < VW; ++c)
        if (FULL || elem(i, c) < N) atomicAdd(S.hist + hslot(key[i * VW + c] >> kSh), 1u);
    group_sync<RG>(g);
    uint32_t b0, below, cnt;
    bool special;
    row_find<RG>(S, g, k, Tr::kHasNan, b0, below, cnt, special);

    if (Tr::kHasNan && special) {
      // a NaN or an infinity is present: the first NaN (in index order) decides
      uint32_t mine = ~0u;
#pragma unroll
      for (int i = 0; i < NI; ++i)
#pragma unroll
        for (int c = 0; c < VW; ++c) {
          const uint32_t e = (uint32_t)elem(i, c);
          if ((FULL || (int)e < N) && Tr::key_is_nan(key[i * VW + c]) && e < mine) mine = e;
        }
      if (mine != ~0u) atomicMin(&S.first_nan, mine);
      group_sync<RG>(g);
      const uint32_t fn = S.first_nan;
      group_sync<RG>(g);
      if (fn != ~0u) {
        if (t == 0) {
          idxs[row] = (int64_t)fn;
          vals[row] = x[row * (int64_t)N + fn];
          S.first_nan = ~0u;
        }
        continue;
      }
    }
    uint32_t r = k - below;

    // ---- compact the bucket's elements as (key << kDig) | index, per warp
    const uint32_t lo = b0 << kSh;
    {
      uint32_t* L = S.list + kRegion * w;
      const uint32_t lt = lanemask_lt();
      uint32_t nw = 0;
#pragma unroll
      for (int i = 0; i < NI; ++i)
#pragma unroll
        for (int c = 0; c < VW; ++c) {
          const uint32_t kk = key[i * VW + c];
          const bool m = (FULL || elem(i, c) < N) && (kk - lo) < (1u << kSh);
          const uint32_t bal = __ballot_sync(0xffffffffu, m);
          if (bal) {
            if (m) L[nw + __popc(bal & lt)] = (kk << kDig) | (uint32_t)elem(i, c);
            nw += __popc(bal);
          }
        }
      if (lane == 0) S.wcnt[w] = nw;
    }
    group_sync<RG>(g);

    uint32_t comp = 0;
    bool owner = false;
    if (cnt <= 32) {
      // one warp: the composite with exactly r smaller composites
      if (w == fw) {
        uint32_t base = 0, v = ~0u;
#pragma unroll
        for (int q = 0; q < RG; ++q) {
          const uint32_t nq = S.wcnt[q];
          if ((uint32_t)lane >= base && (uint32_t)lane < base + nq)
            v = S.list[kRegion * q + (lane - base)];
          base += nq;
        }
        S.tmp[lane] = v;
        __syncwarp();
        uint32_t rank = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint4 o = reinterpret_cast<const uint4*>(S.tmp)[j];
          rank += (o.x < v) + (o.y < v) + (o.z < v) + (o.w < v);
        }
        owner = (uint32_t)lane < cnt && rank == r;
        comp = v;
        __syncwarp();
      }
    } else {
      // radix passes over the per-warp lists, kDig bits at a time from the top
      uint32_t pref = 0;
      uint32_t nq[RG];
#pragma unroll
      for (int q = 0; q < RG; ++q) nq[q] = S.wcnt[q];
#pragma unroll 1
      for (int done = 0; done < 32;) {
        const int wb = (32 - done) < kDig ? (32 - done) : kDig;
        const int sh = 32 - done - wb;
        const uint32_t hmask = done == 0 ? 0u : (~0u << (32 - done));
#pragma unroll
        for (int q = 0; q < RG; ++q)
          for (uint32_t u = t; u < nq[q]; u += RG * 32) {
            const uint32_t cq = S.list[kRegion * q + u];
            if ((cq & hmask) == pref) atomicAdd(S.hist + hslot((cq >> sh) & ((1u << wb) - 1u)), 1u);
          }
        group_sync<RG>(g);
        uint32_t bb, bl, bc;
        bool dummy;
        row_find<RG>(S, g, r, false, bb, bl, bc, dummy);
        r -= bl;
        pref |= bb << sh;
        done += wb;
      }
      comp = pref;
      owner = (t == 0);
    }
    if (owner) {
      const uint32_t e = comp & ((1u << kDig) - 1u);
      const uint32_t kf = lo | (comp >> kDig);
      idxs[row] = (int64_t)e;
      vals[row] = Tr::is_zero_key(kf) ? x[row * (int64_t)N + e] : Tr::from_key(kf);
    }
  }
}

// ---------------------------------------------------------------------------
// rows of 1024 < N <= 2048 of 4-byte elements (16-byte aligned): producer and
// consumer warps
// ---------------------------------------------------------------------------
// Two rates have to be met at once: HBM needs ~64 KiB of reads in flight per
// SM at all times, and each row's selection is a chain of dependent
// shared-memory round trips (scan, compaction, selection) several thousand
// cycles long.  Warps that both load and select a row stall their loads for the
// length of the chain, so the work is split (512 threads, one CTA per SM):
//   producers (4 warps): keep the next kWsPD rows in flight in registers (16
//     elements per thread), stage the current row's words as loaded in slot
//     q % kWsSlots and count them in the slot's histogram of the words' top 11
//     bits (one shift and one shared atomic per element: no key transform),
//     and move on;
//   consumers (kWsSlots warps, row q goes to consumer q % kWsSlots, which owns
//     that slot): scan the histogram in value order (clearing it), compact the
//     selected bin from the staged words, select, and hand the slot back.
// A consumer's row is a chain of dependent shared-memory round trips, so the
// number of consumers (rows being selected at once) sets the rate: 12 slots of
// 16 KiB fill the SM's shared memory, and the producers, with only a shift and
// an atomic per element, need 4 warps.
// The raw top 11 bits order the values once the bins are read in the right
// order: for floats (sign-magnitude) the negative bins 2047..1024 come first,
// in reverse, then 0..1023; for int32 (two's complement) bins 1024..2047, then
// 0..1023.  Bin b of the value order is therefore the top 11 bits of the
// order-preserving key, which the consumer computes only for the few elements
// of the selected bin.  The one bin pair the raw order splits is +0.0 / -0.0
// (with the subnormals of either sign): -0.0 sits in raw bin 1024 and +0.0 in
// raw bin 0, adjacent in value order, so a rank landing in either is resolved
// over both with keys that map -0.0 to +0.0.
// Slots past the end of a shorter row hold the word 0x7fffffff, which lands in
// the last bin of the value order (a NaN pattern for floats, INT_MAX for int32)
// and sorts after every element of the row (after every equal element too, by
// index), so rank k is unchanged; the NaN check allows for them in that bin.
// Hand-offs are mbarriers, each waited on by one role in phase order; waits are
// bounded (one that runs out sets the abort flag, stops every role and is
// counted in g_median_timeouts).
constexpr int kWsSlots = 4;  // = consumer warps (8 or 12 measured slower)
constexpr int kWsPD = 4;     // rows in flight per producer thread (5, 6 measured slower)
constexpr int ws_gcd(int a, int b) { return b == 0 ? a : ws_gcd(b, a % b); }
constexpr int kWsU = kWsSlots / ws_gcd(kWsSlots, kWsPD) * kWsPD;  // producer loop period
constexpr int kWsThreads = 128 + 32 * kWsSlots;
static_assert(kWsU % kWsSlots == 0 && kWsU % kWsPD == 0,
              "row q uses register set q % kWsPD and slot q % kWsSlots");
constexpr int kWsCap = 2048;
constexpr uint32_t kWsPad = 0x7fffffffu;
constexpr uint32_t kMedWaitLimit = 1u << 22;
__device__ unsigned int g_median_timeouts;

struct __align__(128) WsSmem {
  uint32_t raw[kWsSlots][kWsCap];   // the row's words as loaded (padding: kWsPad)
  uint32_t hist[kWsSlots][kWsCap];  // counts per raw bin (top 11 bits of the word)
  unsigned long long list[kWsSlots][32];
  uint32_t ccount[kWsSlots];
  uint64_t full[kWsSlots], empty[kWsSlots];
  uint32_t abort_flag;
};

__device__ __forceinline__ void mbar_arrive1(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar)) : "memory");
}

// Bounded wait; false (with the abort flag set) when it runs out or when
// another role has aborted.
__device__ __forceinline__ bool ws_wait(WsSmem& S, uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kMedWaitLimit; ++i) {
    if (tc::mbar_try_wait(bar, parity)) return true;
    if (*(volatile uint32_t*)&S.abort_flag) return false;
  }
  atomicAdd(&g_median_timeouts, 1u);
  *(volatile uint32_t*)&S.abort_flag = 1;
  return false;
}

// Bin orders of bin_find: kOrdPlain = bins ascending (digit histograms of keys);
// kOrdF32 / kOrdI32 = raw top-11-bit bins of float / int32 words in value order.
constexpr int kOrdPlain = 0, kOrdF32 = 1, kOrdI32 = 2;

// Scan of 2^B bins in value order (the orders above); lane l owns the
// chunks 32 j + l, j < 2^B / 128.  Returns to every lane the raw bin holding
// rank r, the count below it and its count, and zeroes the bins.  With `edge`
// (floats), `special` reports a nonzero count in the first 4 bins of the value
// order or more than npad in the last 4; zp / zn return the counts of raw bins
// 0 and 2^(B-1) (the +0.0 and -0.0 bins) for kOrdF32.
template <int kOrd, int B>
__device__ __forceinline__ void bin_find(uint32_t* hist, uint32_t r, bool edge, uint32_t npad,
                                         uint32_t& bin, uint32_t& below, uint32_t& cnt,
                                         bool& special, uint32_t& zp, uint32_t& zn) {
  constexpr int NG = (1 << B) / 128;  // groups of 128 bins = chunks per lane
  constexpr int HG = NG / 2;
  static_assert(kOrd == kOrdPlain || NG >= 2, "value orders split the groups by sign");
  const int lane = threadIdx.x & 31;
  uint4* hp = reinterpret_cast<uint4*>(hist) + lane;
  uint32_t ls[NG];
#pragma unroll
  for (int j = 0; j < NG; ++j) {
    const uint4 h = hp[32 * j];
    ls[j] = h.x + h.y + h.z + h.w;
  }
  if (kOrd == kOrdF32) {
    zp = hist[0];
    zn = hist[1 << (B - 1)];
  }
  bool sp = false;
  if (kOrd == kOrdF32 && edge && lane == 31) sp = ls[NG - 1] != 0u || ls[HG - 1] != npad;
  special = __any_sync(0xffffffffu, sp);
  uint32_t cum = 0, gbelow = 0;
  int J = -1;
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    const int j = kOrd == kOrdPlain ? g : (kOrd == kOrdF32 ? (g < HG ? NG - 1 - g : g - HG)
                                                           : (g < HG ? g + HG : g - HG));
    const uint32_t G = __reduce_add_sync(0xffffffffu, ls[j]);
    if (J < 0 && r < cum + G) {
      J = j;
      gbelow = cum;
    }
    cum += G;
  }
  if (J < 0) J = 0;  // r beyond the total: not reached for a valid rank
  const bool desc = kOrd == kOrdF32 && J >= HG;
  const uint4 h = hp[32 * J];
  const uint32_t c[4] = {desc ? h.w : h.x, desc ? h.z : h.y, desc ? h.y : h.z, desc ? h.x : h.w};
  const uint32_t tot = c[0] + c[1] + c[2] + c[3];
  uint32_t inc = tot;
  if (desc) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_down_sync(0xffffffffu, inc, o);
      if (lane + o < 32) inc += y;
    }
  } else {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += y;
    }
  }
  const uint32_t rr = r - gbelow;
  const uint32_t exc = inc - tot;
  const bool own = exc <= rr && rr < inc;
  const int ol = __ffs(__ballot_sync(0xffffffffu, own)) - 1;
  uint32_t pb = 0, pbl = 0, pc = 0;
  if (own) {
    uint32_t acc = exc;
    int w = 0;
#pragma unroll
    for (int j = 0; j < 3; ++j)
      if (w == j && rr >= acc + c[j]) {
        acc += c[j];
        w = j + 1;
      }
    uint32_t cw = c[0];
#pragma unroll
    for (int j = 1; j < 4; ++j)
      if (w == j) cw = c[j];
    pb = 128u * J + 4u * lane + (desc ? 3 - w : w);
    pbl = gbelow + acc;
    pc = cw;
  }
  __syncwarp();  // every lane's reads (zp / zn included) before the clear
#pragma unroll
  for (int j = 0; j < NG; ++j) hp[32 * j] = make_uint4(0, 0, 0, 0);
  bin = __shfl_sync(0xffffffffu, pb, ol < 0 ? 0 : ol);
  below = __shfl_sync(0xffffffffu, pbl, ol < 0 ? 0 : ol);
  cnt = __shfl_sync(0xffffffffu, pc, ol < 0 ? 0 : ol);
}

// value-order position of raw bin s (= the top 11 bits of the element's key)
template <typename T>
__device__ __forceinline__ uint32_t ws_pos(uint32_t s) {
  if constexpr (std::is_same<T, float>::value) return s < 1024u ? s + 1024u : 2047u - s;
  else return s ^ 1024u;
}

template <typename T>
__device__ __forceinline__ uint32_t ws_key(uint32_t u) {
  if constexpr (std::is_same<T, float>::value) return KeyTraits<float>::key(__uint_as_float(u));
  else return KeyTraits<T>::key((T)u);
}

template <typename T>
__global__ void __launch_bounds__(kWsThreads, kWsSlots <= 4 ? 2 : 1)
median_ws_kernel(const T* __restrict__ x, T* __restrict__ vals, int64_t* __restrict__ idxs,
                 int64_t M, int N) {
  using Tr = KeyTraits<T>;
  static_assert(sizeof(T) == 4, "4-byte elements");
  constexpr bool kF = std::is_same<T, float>::value;
  constexpr int kOrd = kF ? kOrdF32 : kOrdI32;
  extern __shared__ __align__(128) uint8_t median_smem[];
  WsSmem& S = *reinterpret_cast<WsSmem*>(median_smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t k = (uint32_t)(N - 1) / 2;
  const uint32_t npad = (uint32_t)(kWsCap - N);
  const int64_t rstep = gridDim.x;
  // rows of this CTA: q-th row = blockIdx.x + q * gridDim.x
  const int64_t nq = M > blockIdx.x ? (M - 1 - blockIdx.x) / rstep + 1 : 0;

  for (int j = threadIdx.x; j < kWsSlots * kWsCap / 4; j += blockDim.x)
    reinterpret_cast<uint4*>(&S.hist[0][0])[j] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x < kWsSlots) S.ccount[threadIdx.x] = 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kWsSlots; ++s) {
      tc::mbar_init(&S.full[s], 128);
      tc::mbar_init(&S.empty[s], 32);
    }
    S.abort_flag = 0;
    tc::fence_mbar_init();
  }
  __syncthreads();

  if (warp < 4) {
    // ---------------- producers
    const int t = threadIdx.x;  // 0..127; element (i, c) = (i * 128 + t) * 4 + c
    uint4 rv[kWsPD][4];
    // N is a multiple of 4 (16-byte rows), so a vector is either all in the
    // row or all padding
    auto load_row = [&](int64_t q, uint4 (&dst)[4]) {
      if (q >= nq) return;
      const T* xx = x + (blockIdx.x + q * rstep) * (int64_t)N;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int base = (i * 128 + t) * 4;
        dst[i] = base < N ? ld_global_stream_v4(xx + base)
                          : make_uint4(kWsPad, kWsPad, kWsPad, kWsPad);
      }
    };
#pragma unroll
    for (int j = 0; j < kWsPD; ++j) load_row(j, rv[j]);
    bool stop = false;
    for (int64_t qb = 0; qb < nq && !stop; qb += kWsU) {
#pragma unroll
      for (int j = 0; j < kWsU; ++j) {
        // row qb + j lives in rv[j % kWsPD] and goes to slot j % kWsSlots
        const int64_t q = qb + j;
        if (q >= nq || stop) break;
        uint4 (&cur)[4] = rv[j % kWsPD];
        const int sl = j % kWsSlots;
        const int64_t use = q / kWsSlots;
        if (use > 0 && !ws_wait(S, &S.empty[sl], (uint32_t)(use - 1) & 1u)) {
          stop = true;
          break;
        }
        uint32_t* Rw = S.raw[sl];
#pragma unroll
        for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(Rw + (i * 128 + t) * 4) = cur[i];
        uint32_t* H = S.hist[sl];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          atomicAdd(H + (cur[i].x >> 21), 1u);
          atomicAdd(H + (cur[i].y >> 21), 1u);
          atomicAdd(H + (cur[i].z >> 21), 1u);
          atomicAdd(H + (cur[i].w >> 21), 1u);
        }
        load_row(q + kWsPD, cur);  // the row's registers are free again
        mbar_arrive1(&S.full[sl]);
      }
    }
    return;
  }

  // ---------------- consumers
  const int cw = warp - 4;
  uint32_t* H = S.hist[cw];
  unsigned long long* L = S.list[cw];
  for (int64_t q = cw; q < nq; q += kWsSlots) {
    const int64_t row = blockIdx.x + q * rstep;
    if (!ws_wait(S, &S.full[cw], (uint32_t)(q / kWsSlots) & 1u)) break;
    const uint4* R4 = reinterpret_cast<const uint4*>(S.raw[cw]);
    uint32_t s, below, cnt, z0 = 0, z1024 = 0;
    bool special;
    bin_find<kOrd, 11>(H, k, kF, npad, s, below, cnt, special, z0, z1024);
    bool done = false;
    if (kF && special) {
      // a NaN or an infinity is present: the first NaN (in index order) decides
      uint32_t mine = ~0u;
      for (int i = 0; i < 16; ++i) {
        const int ch = i * 32 + lane;
        const uint4 kv = R4[ch];
        const uint32_t kk[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (4 * ch + c < N && (kk[c] & 0x7fffffffu) > 0x7f800000u)
            mine = min(mine, (uint32_t)(4 * ch + c));
      }
      const uint32_t fn = __reduce_min_sync(0xffffffffu, mine);
      if (fn != ~0u) {
        if (lane == 0) {
          idxs[row] = (int64_t)fn;
          vals[row] = x[row * (int64_t)N + fn];
        }
        done = true;
      }
    }
    if (!done) {
      // The selected bin in key space: prefix P under mask Mk of key - koff.
      uint32_t koff = 0, P, Mk;
      int known;
      if (kF && (s == 0u || s == 1024u)) {
        // +0.0 / -0.0 (and subnormals): value-order bins 1023 and 1024 as one,
        // keys shifted so the pair is the prefix 0 of 10 bits
        if (s == 0u) below -= z1024;
        cnt = z0 + z1024;
        koff = 1023u << 21;
        P = 0u;
        Mk = 0xffc00000u;
        known = 10;
      } else {
        P = ws_pos<T>(s) << 21;
        Mk = 0xffe00000u;
        known = 11;
      }
      uint32_t r = k - below;
      while (cnt > 32 && known < 32) {
        // narrow the bin with the next key bits (this warp's histogram)
        const int nb = (32 - known) < 11 ? (32 - known) : 11;
        const int sh = 32 - known - nb;
        const uint32_t dm = (1u << nb) - 1u;
        for (int i = 0; i < 16; ++i) {
          const uint4 kv = R4[i * 32 + lane];
          const uint32_t kk[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t key = ws_key<T>(kk[c]) - koff;
            if ((key & Mk) == P) atomicAdd(H + ((key >> sh) & dm), 1u);
          }
        }
        __syncwarp();
        uint32_t bb, bl, d0, d1;
        bool unused;
        bin_find<kOrdPlain, 11>(H, r, false, 0, bb, bl, cnt, unused, d0, d1);
        r -= bl;
        P |= bb << sh;
        Mk |= dm << sh;
        known += nb;
      }
      uint32_t e_ans = 0, k_ans = P;
      bool owner = false;
      if (cnt <= 32) {
        // compact the bin as (key << 32 | index): match masks first, then one
        // slot reservation per lane that holds any
        uint32_t mlo = 0, mhi = 0;
        if (known <= 11) {
          // the first pass's bin (or the +-0 pair): compare the words' top bits
          const uint32_t wm = known == 11 ? 0xffe00000u : 0x7fe00000u;
          const uint32_t wv = known == 11 ? s << 21 : 0u;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint4 kv = R4[i * 32 + lane];
            const uint32_t kk[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint32_t bit = ((kk[c] & wm) == wv) ? 1u : 0u;
              if (i < 8) mlo |= bit << (4 * i + c);
              else mhi |= bit << (4 * (i - 8) + c);
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint4 kv = R4[i * 32 + lane];
            const uint32_t kk[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint32_t bit = (((ws_key<T>(kk[c]) - koff) & Mk) == P) ? 1u : 0u;
              if (i < 8) mlo |= bit << (4 * i + c);
              else mhi |= bit << (4 * (i - 8) + c);
            }
          }
        }
        const uint32_t nl = __popc(mlo) + __popc(mhi);
        if (nl) {
          uint32_t pos = atomicAdd(&S.ccount[cw], nl);
          unsigned long long mm = ((unsigned long long)mhi << 32) | mlo;
          const uint32_t* Rw = S.raw[cw];
          while (mm) {
            const int j = __ffsll((long long)mm) - 1;
            mm &= mm - 1;
            const uint32_t e = (uint32_t)(4 * ((j >> 2) * 32 + lane) + (j & 3));
            L[pos++] = ((unsigned long long)(ws_key<T>(Rw[e]) - koff) << 32) | e;
          }
        }
        __syncwarp();
        const unsigned long long v = (uint32_t)lane < cnt ? L[lane] : ~0ull;
        uint32_t rank = 0;
        for (uint32_t j = 0; j < cnt; ++j) rank += L[j] < v ? 1u : 0u;  // cnt: warp-uniform
        owner = (uint32_t)lane < cnt && rank == r;
        e_ans = (uint32_t)v;
        k_ans = (uint32_t)(v >> 32);
        if (lane == 0) S.ccount[cw] = 0;
      } else {
        // all key bits known: the r-th element equal to P in index order
        for (int i = 0; i < 16; ++i) {
          const int ch = i * 32 + lane;
          const uint4 kv = R4[ch];
          const uint32_t kk[4] = {kv.x, kv.y, kv.z, kv.w};
          uint32_t mc = 0;
#pragma unroll
          for (int c = 0; c < 4; ++c) mc += (ws_key<T>(kk[c]) - koff) == P ? 1u : 0u;
          uint32_t inc = mc;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += y;
          }
          const uint32_t total = __shfl_sync(0xffffffffu, inc, 31);
          if (r < total) {
            const uint32_t exc = inc - mc;
            if (exc <= r && r < inc) {
              uint32_t qq = r - exc;
#pragma unroll
              for (int c = 0; c < 4; ++c)
                if ((ws_key<T>(kk[c]) - koff) == P) {
                  if (qq == 0 && !owner) {
                    owner = true;
                    e_ans = (uint32_t)(4 * ch + c);
                  }
                  --qq;
                }
            }
            break;
          }
          r -= total;
        }
      }
      if (owner) {
        const uint32_t kf = k_ans + koff;
        idxs[row] = (int64_t)e_ans;
        vals[row] = Tr::is_zero_key(kf) ? x[row * (int64_t)N + e_ans] : Tr::from_key(kf);
      }
    }
    __syncwarp();
    mbar_arrive1(&S.empty[cw]);  // words and the cleared histogram back to the producers
  }
}


template <typename T>
int launch_ws_rows(const void* x, void* v, int64_t* idx, int64_t M, int N, cudaStream_t st) {
  auto kern = median_ws_kernel<T>;
  const int smem = (int)sizeof(WsSmem);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
    set_error("median: cannot reserve %d bytes of shared memory", smem);
    return FO_ECUDA;
  }
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kWsThreads, smem);
  if (per_sm < 1) per_sm = 1;
  int64_t grid = (int64_t)num_sms() * per_sm;
  if (grid > M) grid = M;
  kern<<<(unsigned)grid, kWsThreads, smem, st>>>((const T*)x, (T*)v, idx, M, N);
  return check_launch("median_ws_kernel");
}

// ---------------------------------------------------------------------------
// one warp per row, the row in registers (4-byte types, N <= 2048)
// ---------------------------------------------------------------------------
// Each lane holds NI words of the row (vector mode: NI / 4 16-byte vectors,
// element (v, c) = (32 v + lane) * 4 + c; scalar mode: element 32 i + lane),
// and the next row's words are loaded while the current row is selected, so a
// warp always has one row in flight.  Per row:
//   1. one shared atomic per element into the warp's histogram of the words'
//      top B bits (no key transform: the bins are read in value order, as in
//      the producer/consumer kernel above);
//   2. the warp scans the histogram (lane l reads the 16-byte chunks 32 j + l,
//      free of bank conflicts) for the bin holding rank k and clears it;
//   3. the bin's elements are compacted from the registers as (key << 32 |
//      index) composites and ranked; more than 32 go through further digit
//      passes over the registers.
// Shared-memory traffic per row is the histogram alone (atomics, one read, one
// clear): the row itself never passes through shared memory.
template <int B>
struct __align__(16) WarpSmem {
  uint32_t hist[1 << B];
  unsigned long long list[32];
  uint32_t ccount;
  uint32_t pad_[3];
};

// value-order position of raw bin s of 2^B (= the top B bits of the key)
template <typename T, int B>
__device__ __forceinline__ uint32_t bin_pos(uint32_t s) {
  constexpr uint32_t H = 1u << (B - 1);
  if constexpr (std::is_same<T, float>::value) return s < H ? s + H : 2 * H - 1 - s;
  else return s ^ H;
}

// The words of a row in a lane: NV 16-byte vectors (VW = 4) or NI scalars.
template <int NI, int VW>
struct RowRegs {
  uint32_t w[NI];
};

template <typename T, int NI, int VW>
__device__ __forceinline__ void wr_load(const T* __restrict__ xr, int N, int lane,
                                        RowRegs<NI, VW>& R) {
  if constexpr (VW == 4) {
#pragma unroll
    for (int v = 0; v < NI / 4; ++v) {
      const int base = (32 * v + lane) * 4;
      const uint4 u = base < N ? ld_global_stream_v4(xr + base)
                               : make_uint4(kWsPad, kWsPad, kWsPad, kWsPad);
      R.w[4 * v] = u.x;
      R.w[4 * v + 1] = u.y;
      R.w[4 * v + 2] = u.z;
      R.w[4 * v + 3] = u.w;
    }
  } else {
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(xr);
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int e = 32 * i + lane;
      R.w[i] = e < N ? __ldg(xw + e) : kWsPad;
    }
  }
}

// element index of word i of this lane
template <int VW>
__device__ __forceinline__ uint32_t wr_elem(int i, int lane) {
  if constexpr (VW == 4) return (uint32_t)((32 * (i >> 2) + lane) * 4 + (i & 3));
  else return (uint32_t)(32 * i + lane);
}

template <typename T, int NI, int VW, int B>
__device__ __forceinline__ void wr_select(const T* __restrict__ x, T* __restrict__ vals,
                                          int64_t* __restrict__ idxs, int64_t row, int N,
                                          const RowRegs<NI, VW>& R, WarpSmem<B>& S) {
  using Tr = KeyTraits<T>;
  constexpr bool kF = std::is_same<T, float>::value;
  constexpr int kOrd = kF ? kOrdF32 : kOrdI32;
  constexpr int SH = 32 - B;
  const int lane = threadIdx.x & 31;
  const uint32_t k = (uint32_t)(N - 1) / 2;
  const uint32_t npad = (uint32_t)(32 * NI - N);

#pragma unroll
  for (int i = 0; i < NI; ++i) atomicAdd(S.hist + (R.w[i] >> SH), 1u);
  __syncwarp();
  uint32_t s, below, cnt, zp = 0, zn = 0;
  bool special;
  bin_find<kOrd, B>(S.hist, k, kF, npad, s, below, cnt, special, zp, zn);
  if (kF && special) {
    // a NaN or an infinity may be present: the first NaN (in index order) decides
    uint32_t mine = ~0u;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const uint32_t e = wr_elem<VW>(i, lane);
      if ((R.w[i] & 0x7fffffffu) > 0x7f800000u && e < (uint32_t)N && e < mine) mine = e;
    }
    const uint32_t fn = __reduce_min_sync(0xffffffffu, mine);
    if (fn != ~0u) {
      if (lane == 0) {
        idxs[row] = (int64_t)fn;
        vals[row] = x[row * (int64_t)N + fn];
      }
      return;
    }
  }
  // the selected bin in key space: prefix P under mask Mk of key - koff
  uint32_t koff = 0, P, Mk, wm, wv;
  int known;
  if (kF && (s == 0u || s == (1u << (B - 1)))) {
    // +0.0 / -0.0 (and the smallest values of either sign): value-order bins
    // 2^(B-1) - 1 and 2^(B-1) as one, keys shifted so the pair is a prefix
    if (s == 0u) below -= zn;
    cnt = zp + zn;
    koff = ((1u << (B - 1)) - 1u) << SH;
    P = 0u;
    Mk = ~0u << (SH + 1);
    known = B - 1;
    wm = 0x7fffffffu & (~0u << SH);
    wv = 0u;
  } else {
    P = bin_pos<T, B>(s) << SH;
    Mk = ~0u << SH;
    known = B;
    wm = ~0u << SH;
    wv = s << SH;
  }
  uint32_t r = k - below;
  while (cnt > 32 && known < 32) {
    // narrow the bin with the next key bits (histogram of the next digit)
    const int nb = (32 - known) < B ? (32 - known) : B;
    const int sh = 32 - known - nb;
    const uint32_t dm = (1u << nb) - 1u;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const uint32_t key = ws_key<T>(R.w[i]) - koff;
      if ((key & Mk) == P) atomicAdd(S.hist + ((key >> sh) & dm), 1u);
    }
    __syncwarp();
    uint32_t bb, bl, d0, d1;
    bool unused;
    bin_find<kOrdPlain, B>(S.hist, r, false, 0, bb, bl, cnt, unused, d0, d1);
    r -= bl;
    P |= bb << sh;
    Mk |= dm << sh;
    known += nb;
    wm = 0u;  // matches are by key from here on
  }
  uint32_t e_ans = 0, k_ans = P;
  bool owner = false;
  if (cnt <= 32) {
    // compact the bin as (key << 32 | index)
    uint32_t m[(NI + 31) / 32] = {};
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const bool hit = wm ? ((R.w[i] & wm) == wv) : (((ws_key<T>(R.w[i]) - koff) & Mk) == P);
      if (hit) m[i >> 5] |= 1u << (i & 31);
    }
    uint32_t nl = 0;
#pragma unroll
    for (int q = 0; q < (NI + 31) / 32; ++q) nl += __popc(m[q]);
    if (nl) {
      uint32_t pos = atomicAdd(&S.ccount, nl);
#pragma unroll
      for (int i = 0; i < NI; ++i)
        if (m[i >> 5] & (1u << (i & 31)))
          S.list[pos++] = ((unsigned long long)(ws_key<T>(R.w[i]) - koff) << 32) | wr_elem<VW>(i, lane);
    }
    __syncwarp();
    const unsigned long long v = (uint32_t)lane < cnt ? S.list[lane] : ~0ull;
    uint32_t rank = 0;
    for (uint32_t j = 0; j < cnt; ++j) rank += S.list[j] < v ? 1u : 0u;  // cnt: warp-uniform
    owner = (uint32_t)lane < cnt && rank == r;
    e_ans = (uint32_t)v;
    k_ans = (uint32_t)(v >> 32);
    __syncwarp();
    if (lane == 0) S.ccount = 0;
  } else {
    // all key bits known: the r-th element equal to P in index order, walking
    // the words in index order (vector v of all lanes, then v + 1)
    // (no early exit: every word index stays a compile-time constant)
    constexpr int NV = VW == 4 ? NI / 4 : NI;
    bool found = false;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      uint32_t mc = 0;
#pragma unroll
      for (int c = 0; c < VW; ++c) mc += (ws_key<T>(R.w[v * VW + c]) - koff) == P ? 1u : 0u;
      uint32_t inc = mc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
      }
      const uint32_t total = __shfl_sync(0xffffffffu, inc, 31);
      if (!found) {
        if (r < total) {
          found = true;
          const uint32_t exc = inc - mc;
          if (exc <= r && r < inc) {
            uint32_t qq = r - exc;
#pragma unroll
            for (int c = 0; c < VW; ++c)
              if ((ws_key<T>(R.w[v * VW + c]) - koff) == P) {
                if (qq == 0 && !owner) {
                  owner = true;
                  e_ans = wr_elem<VW>(v * VW + c, lane);
                }
                --qq;
              }
          }
        } else {
          r -= total;
        }
      }
    }
  }
  if (owner) {
    const uint32_t kf = k_ans + koff;
    idxs[row] = (int64_t)e_ans;
    vals[row] = Tr::is_zero_key(kf) ? x[row * (int64_t)N + e_ans] : Tr::from_key(kf);
  }
}

constexpr int kWrWarps = 4;  // warps (rows) per CTA


template <typename T, int NI, int VW, int B, int MINB, int D>
__global__ void __launch_bounds__(32 * kWrWarps, MINB)
median_warp_kernel(const T* __restrict__ x, T* __restrict__ vals, int64_t* __restrict__ idxs,
                   int64_t M, int N) {
  extern __shared__ __align__(16) uint8_t median_smem[];
  WarpSmem<B>& S = reinterpret_cast<WarpSmem<B>*>(median_smem)[threadIdx.x >> 5];
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < (1 << B) / 128; ++j)
    reinterpret_cast<uint4*>(S.hist)[32 * j + lane] = make_uint4(0, 0, 0, 0);
  if (lane == 0) S.ccount = 0;
  __syncwarp();
  const int64_t stride = (int64_t)gridDim.x * kWrWarps;
  int64_t row = (int64_t)blockIdx.x * kWrWarps + (threadIdx.x >> 5);
  // a ring of D register sets: the next D - 1 rows load while one is selected
  RowRegs<NI, VW> ring[D];
#pragma unroll
  for (int d = 0; d < D - 1; ++d)
    if (row + d * stride < M) wr_load<T, NI, VW>(x + (row + d * stride) * (int64_t)N, N, lane, ring[d]);
  for (; row < M; row += D * stride) {
#pragma unroll
    for (int d = 0; d < D; ++d) {
      const int64_t rd = row + d * stride;
      if (rd >= M) break;
      const int64_t rl = rd + (D - 1) * stride;
      if (rl < M) wr_load<T, NI, VW>(x + rl * (int64_t)N, N, lane, ring[(d + D - 1) % D]);
      wr_select<T, NI, VW, B>(x, vals, idxs, rd, N, ring[d], S);
    }
  }
}

template <typename T, int NI, int VW, int B, int MINB, int D>
int launch_warp_rows(const void* x, void* v, int64_t* idx, int64_t M, int N, cudaStream_t st) {
  auto kern = median_warp_kernel<T, NI, VW, B, MINB, D>;
  const int smem = (int)(kWrWarps * sizeof(WarpSmem<B>));
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
    set_error("median: cannot reserve %d bytes of shared memory", smem);
    return FO_ECUDA;
  }
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 32 * kWrWarps, smem);
  if (per_sm < 1) per_sm = 1;
  const int64_t need = (M + kWrWarps - 1) / kWrWarps;
  int64_t grid = (int64_t)num_sms() * per_sm;
  if (grid > need) grid = need;
  kern<<<(unsigned)grid, 32 * kWrWarps, smem, st>>>((const T*)x, (T*)v, idx, M, N);
  return check_launch("median_warp_kernel");
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
// global median of n >= 2^20 elements: the whole grid per radix pass
// ---------------------------------------------------------------------------
// Every CTA owns a contiguous chunk of x.  Per pass, each CTA histograms the
// digit of its chunk's elements that match the prefix selected so far into
// shared memory and adds its non-empty bins to a global histogram; the last CTA
// of the pass to finish (threadfence + ticket) then picks the bin holding rank
// r and clears the histogram, so a pass is one launch.  After the last
// pass the key is known and gives the value, except for the key that +0.0 and
// -0.0 share: then each CTA counts its zeros and one CTA walks the chunk holding
// the r-th zero in index order and returns it, sign included.  The first NaN
// (lowest index) decides an input holding any NaN.
constexpr int kGmThreads = 512;
constexpr int kGmBins = 2048;
constexpr int kGmMaxCtas = 1024;
static_assert(kGmMaxCtas <= 2 * kGmThreads, "gm_pick_block scans two counts per thread");
constexpr int64_t kGmMinN = (int64_t)1 << 20;

struct GmState {
  unsigned long long prefix, mask, r, first_nan;
  unsigned long long bin_cnt;  // elements in the bin selected by the last pass
  unsigned int ovf;            // 1: the candidates of pass 1 were not (all) kept
  unsigned int ticket;         // CTAs of the current kernel that finished (last one finishes up)
};

// Geometry of the grid path: G CTAs with chunks of a multiple of 2048 elements
// (every chunk start 16-byte aligned) and, per CTA, a region of R candidate
// keys: pass 1 keeps the keys of the bin selected by pass 0 there, and later
// passes read those instead of x when every CTA's candidates fit.
struct GmGeo {
  int64_t G, chunk, R;
};
inline GmGeo gm_geo(int64_t n) {
  int64_t G = (int64_t)num_sms() * 2;
  if (G > kGmMaxCtas) G = kGmMaxCtas;
  const int64_t chunk = ((n + G - 1) / G + 2047) / 2048 * 2048;
  G = (n + chunk - 1) / chunk;
  const int64_t R = chunk < 8192 ? chunk : 8192;
  return {G, chunk, R};
}
// workspace: state (256 B) | histogram | per-CTA counts | per-CTA candidate
// counts | candidate regions (8 bytes per key, whatever the key width)
constexpr int64_t kGmCandOff = 256 + 4 * (kGmBins + 2 * kGmMaxCtas);

// Calls f(j, x[j]) for every j in [j0, j1) of the calling CTA.  When x + j0 is
// 16-byte aligned: 16-byte loads in batches of 4 per thread, software-pipelined
// (the next batch is in flight while the current one is processed); element
// loads for the ragged end, and for the whole range otherwise.
// POL: 0 default L2 policy; 1 evict_last (pass 0: x stays in L2 for pass 1);
// 2 evict_first (pass 1: the last read of x, which also demotes the lines
// pass 0 kept).
template <typename T, int POL = 0, typename F>
__device__ __forceinline__ void gm_for_chunk(const T* __restrict__ x, int64_t j0, int64_t j1, F&& f) {
  constexpr int E = 16 / (int)sizeof(T);
  constexpr int U = 4;
  constexpr int64_t kStep = (int64_t)U * kGmThreads;
  int64_t js = j0;
  if ((reinterpret_cast<uintptr_t>(x + j0) & 15) == 0) {
    const int64_t nv = (j1 - j0) / E;
    const uint4* __restrict__ xv = reinterpret_cast<const uint4*>(x + j0);
    const uint64_t pol = POL == 1 ? l2_policy_evict_last() : l2_policy_evict_first();
    auto load = [&](uint4* r, int64_t v) {
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (v + u * kGmThreads < nv)
          r[u] = POL == 0 ? __ldg(xv + v + u * kGmThreads)
                          : ld_global_hint_v4(xv + v + u * kGmThreads, pol);
    };
    auto proc = [&](const uint4* r, int64_t v) {
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (v + u * kGmThreads < nv) {
          T e[E];
          memcpy(e, &r[u], 16);
#pragma unroll
          for (int i = 0; i < E; ++i) f(j0 + (v + u * kGmThreads) * E + i, e[i]);
        }
    };
    uint4 ra[U], rb[U];
    int64_t v = threadIdx.x;
    if (v < nv) load(ra, v);
    while (v < nv) {
      if (v + kStep < nv) load(rb, v + kStep);
      proc(ra, v);
      v += kStep;
      if (v >= nv) break;
      if (v + kStep < nv) load(ra, v + kStep);
      proc(rb, v);
      v += kStep;
    }
    js = j0 + nv * E;
  }
  for (int64_t j = js + threadIdx.x; j < j1; j += kGmThreads) f(j, x[j]);
}

__global__ void gm_init_kernel(GmState* s, uint32_t* hist, int64_t k) {
  if (threadIdx.x == 0) {
    s->prefix = 0;
    s->mask = 0;
    s->r = (unsigned long long)k;
    s->first_nan = ~0ull;
    s->bin_cnt = 0;
    s->ovf = 0;
    s->ticket = 0;
  }
  for (int j = threadIdx.x; j < kGmBins; j += blockDim.x) hist[j] = 0;
}

// True in exactly one CTA of the grid: the last to get here, after every CTA's
// global writes before this point are visible to it (threadfence + ticket).
// The ticket is reset for the next kernel.
__device__ __forceinline__ bool gm_last_cta(GmState* s) {
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    s_last = atomicAdd(&s->ticket, 1u) == gridDim.x - 1;
    if (s_last) s->ticket = 0;
  }
  __syncthreads();
  if (s_last) __threadfence();
  return s_last != 0;
}

// The bin holding rank r (kGmThreads threads, 4 bins each), run by the last CTA
// of a histogram pass; clears the histogram for the next pass.
template <typename T>
__device__ __forceinline__ void gm_find_block(GmState* s, uint32_t* hist, int p,
                                              const T* __restrict__ x, T* __restrict__ value) {
  using K = typename KeyTraits<T>::K;
  using D = Digits<K>;
  static_assert(kGmBins == 4 * kGmThreads, "4 bins per thread");
  __shared__ uint32_t fsum[kGmThreads / 32];
  __shared__ uint32_t f_bin, f_below, f_cnt;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  uint32_t c[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) c[i] = __ldcg(hist + 4 * tid + i);
#pragma unroll
  for (int i = 0; i < 4; ++i) hist[4 * tid + i] = 0;
  const unsigned long long fnan = *(volatile unsigned long long*)&s->first_nan;
  if (fnan != ~0ull) {
    // a NaN decides (pass 0 looked at every element): its value, as stored
    if (tid == 0 && p == 0) *value = x[fnan];
    return;
  }
  const uint32_t tot = c[0] + c[1] + c[2] + c[3];
  uint32_t inc = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) fsum[wid] = inc;
  __syncthreads();
  uint32_t off = 0;
  for (int q = 0; q < wid; ++q) off += fsum[q];
  const uint64_t exc = (uint64_t)off + inc - tot;
  const uint64_t r = *(volatile unsigned long long*)&s->r;
  if (exc <= r && r < exc + tot) {
    uint64_t acc = exc;
    int w = 0;
#pragma unroll
    for (int i = 0; i < 3; ++i)
      if (w == i && r >= acc + c[i]) {
        acc += c[i];
        w = i + 1;
      }
    uint32_t cw = c[0];
#pragma unroll
    for (int i = 1; i < 4; ++i)
      if (w == i) cw = c[i];
    f_bin = 4 * tid + w;
    f_below = (uint32_t)acc;
    f_cnt = cw;
  }
  __syncthreads();
  if (tid == 0) {
    const int sh = D::shift(p);
    const uint32_t dmask = (1u << D::width(p)) - 1u;
    s->r = r - f_below;
    s->bin_cnt = f_cnt;
    s->prefix |= (unsigned long long)((K)f_bin << sh);
    s->mask |= (unsigned long long)((K)dmask << sh);
    // after the last pass the key is known: it gives the value unless it is
    // the key +0.0 and -0.0 share (then gm_count_kernel picks the element)
    const K key = (K)s->prefix;
    if (p == D::kPasses - 1 && !KeyTraits<T>::is_zero_key(key)) *value = KeyTraits<T>::from_key(key);
    __threadfence();
  }
}

// MODE 0: the first pass (every element counts; NaNs are looked for).
// MODE 1: the second pass over x; also keeps the keys of the bin selected by
//   pass 0 in this CTA's candidate region (when that bin fits all regions).
// MODE 2: later passes; over this CTA's candidates when every CTA kept all of
//   its own, else over x.
template <typename T, int MODE>
__global__ void __launch_bounds__(kGmThreads)
gm_hist_kernel(const T* __restrict__ x, int64_t n, int64_t chunk, GmState* s,
               uint32_t* __restrict__ hist, int p, typename KeyTraits<T>::K* __restrict__ cand,
               uint32_t* __restrict__ ncand, int64_t R, int64_t G, T* __restrict__ value) {
  using Tr = KeyTraits<T>;
  using K = typename Tr::K;
  using D = Digits<K>;
  __shared__ uint32_t h[kGmBins];
  __shared__ uint32_t s_nc;
  // a NaN found by pass 0 decides: every CTA of a later pass returns at once
  // (all of them, so no ticket is taken and none is left over)
  if (MODE > 0 && *(volatile unsigned long long*)&s->first_nan != ~0ull) return;
  const K prefix = (K)s->prefix, mask = (K)s->mask;
  const int sh = D::shift(p);
  const uint32_t nb = 1u << D::width(p), dmask = nb - 1u;
  for (uint32_t j = threadIdx.x; j < nb; j += kGmThreads) h[j] = 0;
  if (threadIdx.x == 0) s_nc = 0;
  __syncthreads();
  const int64_t j0 = (int64_t)blockIdx.x * chunk;
  const int64_t j1 = (j0 + chunk < n) ? j0 + chunk : n;
  const int lane = threadIdx.x & 31;
  K* mine = cand + blockIdx.x * R;
  unsigned long long my_nan = ~0ull;
  if (MODE == 0) {
    gm_for_chunk<T, 1>(x, j0, j1, [&](int64_t j, T v) {
      if (Tr::isnan_(v) && (unsigned long long)j < my_nan) my_nan = (unsigned long long)j;
      atomicAdd(h + ((uint32_t)(Tr::key(v) >> sh) & dmask), 1u);
    });
    if (my_nan != ~0ull) atomicMin(&s->first_nan, my_nan);
  } else if (MODE == 1) {
    const bool keep = s->bin_cnt <= (unsigned long long)(G * R);
    gm_for_chunk<T, 2>(x, j0, j1, [&](int64_t, T v) {
      const K kk = Tr::key(v);
      if ((kk & mask) == prefix) {
        atomicAdd(h + ((uint32_t)(kk >> sh) & dmask), 1u);
        if (keep) {  // append to this CTA's region, one shared atomic per group of lanes
          const unsigned am = __activemask();
          const int lead = __ffs(am) - 1;
          uint32_t base = 0;
          if (lane == lead) base = atomicAdd(&s_nc, (uint32_t)__popc(am));
          base = __shfl_sync(am, base, lead);
          const uint32_t q = base + (uint32_t)__popc(am & ((1u << lane) - 1u));
          if (q < (uint32_t)R) mine[q] = kk;
        }
      }
    });
    __syncthreads();
    if (threadIdx.x == 0) {
      ncand[blockIdx.x] = s_nc;
      if (!keep || s_nc > (uint32_t)R) s->ovf = 1u;
    }
  } else if (!*(volatile unsigned int*)&s->ovf) {
    const uint32_t m = ncand[blockIdx.x];
    for (uint32_t q = threadIdx.x; q < m; q += kGmThreads) {
      const K kk = mine[q];
      if ((kk & mask) == prefix) atomicAdd(h + ((uint32_t)(kk >> sh) & dmask), 1u);
    }
  } else {
    gm_for_chunk<T>(x, j0, j1, [&](int64_t, T v) {
      const K kk = Tr::key(v);
      if ((kk & mask) == prefix) atomicAdd(h + ((uint32_t)(kk >> sh) & dmask), 1u);
    });
  }
  __syncthreads();
  for (uint32_t j = threadIdx.x; j < nb; j += kGmThreads)
    if (h[j]) atomicAdd(hist + j, h[j]);
  // the last CTA of the pass picks the bin (no separate launch)
  if (gm_last_cta(s)) gm_find_block<T>(s, hist, p, x, value);
}

// One CTA: the chunk holding the r-th element with the selected key, then the
// element itself in index order.
template <typename T>
__device__ __forceinline__ void gm_pick_block(const T* __restrict__ x, int64_t n, int64_t chunk,
                                              const GmState* s, const uint32_t* __restrict__ cnt,
                                              int G, T* __restrict__ value) {
  using Tr = KeyTraits<T>;
  using K = typename Tr::K;
  __shared__ uint32_t wsum[kGmThreads / 32];
  __shared__ int s_cta;
  __shared__ unsigned long long s_r;
  __shared__ long long s_found;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const K key = (K)s->prefix;
  // +0.0 and -0.0 share the key: the chunk holding the r-th zero, from a
  // block-wide inclusive scan of the per-CTA counts (two per thread).
  __shared__ unsigned long long wtot[kGmThreads / 32];
  const unsigned long long r0 = s->r;
  const uint32_t a0 = (2 * tid < G) ? __ldcg(cnt + 2 * tid) : 0u;
  const uint32_t a1 = (2 * tid + 1 < G) ? __ldcg(cnt + 2 * tid + 1) : 0u;
  unsigned long long inc = (unsigned long long)a0 + a1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) wtot[wid] = inc;
  if (tid == 0) {
    s_cta = G - 1;
    s_r = 0;
    s_found = -1;
  }
  __syncthreads();
  unsigned long long before = 0;
  for (int q = 0; q < wid; ++q) before += wtot[q];
  const unsigned long long ex = before + inc - a0 - a1;  // zeros in the chunks before 2*tid
  if (r0 >= ex && r0 < ex + a0) {
    s_cta = 2 * tid;
    s_r = r0 - ex;
  } else if (r0 >= ex + a0 && r0 < ex + a0 + a1) {
    s_cta = 2 * tid + 1;
    s_r = r0 - ex - a0;
  }
  __syncthreads();
  const int64_t j0 = (int64_t)s_cta * chunk;
  const int64_t j1 = (j0 + chunk < n) ? j0 + chunk : n;
  unsigned long long r = s_r;
  for (int64_t base = j0; base < j1; base += kGmThreads) {
    const int64_t j = base + tid;
    const bool m = j < j1 && Tr::key(x[j]) == key;
    const uint32_t bal = __ballot_sync(0xffffffffu, m);
    if (lane == 0) wsum[wid] = __popc(bal);
    __syncthreads();
    uint32_t off = 0, tot = 0;
    for (int q = 0; q < kGmThreads / 32; ++q) {
      const uint32_t c = wsum[q];
      if (q < wid) off += c;
      tot += c;
    }
    const uint32_t rank = off + __popc(bal & ((1u << lane) - 1u));
    if (m && (unsigned long long)rank == r) s_found = j;
    __syncthreads();
    if (s_found >= 0 || r < tot) break;
    r -= tot;
  }
  if (tid == 0) *value = s_found >= 0 ? x[s_found] : x[j0];
}


// Only when the key is the one +0.0 and -0.0 share (the value was written
// otherwise): each CTA counts the zeros of its chunk, and the last CTA picks the
// r-th zero in index order (gm_pick_block).
template <typename T>
__global__ void __launch_bounds__(kGmThreads)
gm_count_kernel(const T* __restrict__ x, int64_t n, int64_t chunk, GmState* s,
                uint32_t* __restrict__ cnt, T* __restrict__ value) {
  using Tr = KeyTraits<T>;
  using K = typename Tr::K;
  __shared__ uint32_t red[kGmThreads / 32];
  if (s->first_nan != ~0ull) return;
  const K key = (K)s->prefix;
  if (!Tr::is_zero_key(key)) return;  // the key alone gave the value
  const int64_t j0 = (int64_t)blockIdx.x * chunk;
  const int64_t j1 = (j0 + chunk < n) ? j0 + chunk : n;
  uint32_t c = 0;
  gm_for_chunk<T>(x, j0, j1, [&](int64_t, T v) { c += (Tr::key(v) == key) ? 1u : 0u; });
  c = __reduce_add_sync(0xffffffffu, c);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t t = 0;
    for (int q = 0; q < kGmThreads / 32; ++q) t += red[q];
    cnt[blockIdx.x] = t;
  }
  if (gm_last_cta(s)) gm_pick_block<T>(x, n, chunk, s, cnt, (int)gridDim.x, value);
}

template <typename T>
int launch_grid_median(const void* xv, void* value, int64_t n, void* ws, cudaStream_t st) {
  using K = typename KeyTraits<T>::K;
  const T* x = (const T*)xv;
  GmState* s = reinterpret_cast<GmState*>(ws);
  uint32_t* hist = reinterpret_cast<uint32_t*>((char*)ws + 256);
  uint32_t* cnt = hist + kGmBins;
  uint32_t* ncand = cnt + kGmMaxCtas;
  K* cand = reinterpret_cast<K*>((char*)ws + kGmCandOff);
  const GmGeo geo = gm_geo(n);
  const int64_t G = geo.G, chunk = geo.chunk, R = geo.R;
  // one launch per pass: its last CTA picks the bin (and, after the last pass,
  // writes the value); the count kernel does work only for the +-0 key
  T* out = (T*)value;
  gm_init_kernel<<<1, 256, 0, st>>>(s, hist, (n - 1) / 2);
  for (int p = 0; p < Digits<K>::kPasses; ++p) {
    if (p == 0)
      gm_hist_kernel<T, 0><<<(unsigned)G, kGmThreads, 0, st>>>(x, n, chunk, s, hist, p, cand,
                                                               ncand, R, G, out);
    else if (p == 1)
      gm_hist_kernel<T, 1><<<(unsigned)G, kGmThreads, 0, st>>>(x, n, chunk, s, hist, p, cand,
                                                               ncand, R, G, out);
    else
      gm_hist_kernel<T, 2><<<(unsigned)G, kGmThreads, 0, st>>>(x, n, chunk, s, hist, p, cand,
                                                               ncand, R, G, out);
  }
  gm_count_kernel<T><<<(unsigned)G, kGmThreads, 0, st>>>(x, n, chunk, s, cnt, out);
  return check_launch("global median");
}

// ---------------------------------------------------------------------------
// dispatch
// ---------------------------------------------------------------------------
template <typename T, int RG, int VW, bool FULL>
int launch_rows(const void* x, void* v, int64_t* idx, int64_t M, int N, cudaStream_t st) {
  constexpr int GPC = 8 / RG;  // row groups per CTA (256 threads)
  auto kern = median_rows_kernel<T, RG, VW, FULL, GPC>;
  const int smem = (int)(GPC * sizeof(RowSmem<RG>));
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
  return check_launch("median_rows_kernel");
}

template <typename T, int RG, int VW>
int launch_rows_n(const void* x, void* v, int64_t* idx, int64_t M, int N, cudaStream_t st) {
  if constexpr (VW > 1) {
    if (N == RowGeom<RG>::kCap) return launch_rows<T, RG, VW, true>(x, v, idx, M, N, st);
  }
  return launch_rows<T, RG, VW, false>(x, v, idx, M, N, st);
}

// Row length -> group width RG (warps); 16 elements per thread.
template <typename T>
int dispatch_rows(const void* x, void* v, int64_t* idx, int64_t M, int N, bool vec,
                  cudaStream_t st) {
  constexpr int VWV = 16 / sizeof(T);
  if (vec) {
    if (N <= 512) return launch_rows_n<T, 1, VWV>(x, v, idx, M, N, st);
    if (N <= 1024) return launch_rows_n<T, 2, VWV>(x, v, idx, M, N, st);
    return launch_rows_n<T, 4, VWV>(x, v, idx, M, N, st);
  }
  if (N <= 512) return launch_rows_n<T, 1, 1>(x, v, idx, M, N, st);
  if (N <= 1024) return launch_rows_n<T, 2, 1>(x, v, idx, M, N, st);
  return launch_rows_n<T, 4, 1>(x, v, idx, M, N, st);
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
    if constexpr (sizeof(T) == 4) {
      if (vec && N > 1024) return launch_ws_rows<T>(x, v, idx, M, (int)N, st);
      // rows of 256 < N <= 384: one warp per row, 9 or 12 words per lane,
      // 9-bit bins (measured against the row-group kernel: 0.75x the time at
      // N = 257, 0.82x at 300, 0.96x at 400 and 1.12x at 512, where the
      // row-group kernel keeps its 16-byte loads; a deeper register ring and
      // 8- or 10-bit bins measured slower)
      if (N > 256 && N <= 288) return launch_warp_rows<T, 9, 1, 9, 8, 2>(x, v, idx, M, (int)N, st);
      if (N > 256 && N <= 384) return launch_warp_rows<T, 12, 1, 9, 7, 2>(x, v, idx, M, (int)N, st);
    }
    return dispatch_rows<T>(x, v, idx, M, (int)N, vec, st);
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

extern "C" int fo_median_timeouts(unsigned int* count) {
  clear_error();
  FO_CHECK_ARG(count, "fo_median_timeouts: null pointer");
  if (cudaMemcpyFromSymbol(count, g_median_timeouts, sizeof(unsigned int)) != cudaSuccess) {
    set_error("fo_median_timeouts: cannot read the device counter");
    return FO_ECUDA;
  }
  return FO_OK;
}

extern "C" int fo_median_all_workspace_bytes(int64_t n, int64_t* bytes) {
  clear_error();
  FO_CHECK_ARG(bytes && n >= 0, "fo_median_all_workspace_bytes: bad argument");
  // small n: the index of the selected element (one CTA); large n: the grid
  // path's state, histogram, per-CTA counts and candidate regions
  if (n >= kGmMinN) {
    const GmGeo geo = gm_geo(n);
    *bytes = kGmCandOff + geo.G * geo.R * 8;
  } else {
    *bytes = 8;
  }
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
  if (n >= kGmMinN && n < ((int64_t)1 << 32)) {
    int64_t need = 0;
    fo_median_all_workspace_bytes(n, &need);
    if (ws_bytes < need) {
      set_error("median: workspace of %lld bytes required", (long long)need);
      return FO_EWORKSPACE;
    }
    switch (dtype) {
      case FO_F32: return launch_grid_median<float>(x, value, n, workspace, st);
      case FO_F16: return launch_grid_median<__half>(x, value, n, workspace, st);
      case FO_BF16: return launch_grid_median<__nv_bfloat16>(x, value, n, workspace, st);
      case FO_I32: return launch_grid_median<int32_t>(x, value, n, workspace, st);
      case FO_I64: return launch_grid_median<int64_t>(x, value, n, workspace, st);
    }
  }
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
