// chunk_gated_delta_rule on sm_100a tensor cores (tcgen05), D = 128, chunk C = 64.
//
// Recurrence (reference _ref_forward, operators/chunk_gated_delta_rule.py:291-308):
//   h_t = g_t h_{t-1} + beta_t (v_t - h_{t-1} k_t) k_t^T ,  o_t = h_t q_t
// h is [D_v, D_k].  The erase term uses the UNGATED h_{t-1}, i.e. the transition
// is g_t I - beta_t k_t k_t^T.
//
// Chunk algebra (derived from the recurrence; entry state S, tokens t = 0..C-1,
// gamma_t = prod_{r<=t} g_r inside the chunk, ratio(t,s) = gamma_t / gamma_s):
//   u_t = v_t - h_{t-1} k_t  satisfies  (I + A) U = V - diag(gamma_{t-1}) K S^T
//     with A[t,s] = ratio(t-1,s) beta_s (k_t . k_s) for s < t (strictly lower).
//   T = (I + A)^-1 (unit lower triangular), W = T diag(gamma_{s-1}) K, U0 = T V:
//     U = U0 - W S^T
//   O   = diag(gamma_t) Q S^T + P U,   P[t,s] = ratio(t,s) beta_s (q_t . k_s), s <= t
//   S'  = gamma_{C-1} S + U^T Kt,      Kt[s,:] = ratio(C-1,s) beta_s k_s
// Gate ratios are exp of differences of in-chunk prefix sums of log|g|, with the
// sign from the parity of negative gates and an exact 0 when a zero gate lies
// between s and t (g = 0 resets the state, as in the reference test suite).
//
// Every product is a tcgen05.mma with M = 128 by computing transposes: the rows
// of U^T, O^T and of the state are the D_v = 128 value channels.  Per chunk:
//   (a) [Q;K] K^T          M=128 N=64  K=128   -> QK^T and KK^T in one MMA
//   (b) W^T  = (gK)^T T^T   M=128 N=64  K=64
//   (c) U^T  = V^T T^T      M=128 N=64  K=64
//   (d) U^T += S (-W)^T     M=128 N=64  K=128   (needs the state)
//   (e) O^T  = S (gQ)^T     M=128 N=64  K=128   (needs the state)
//   (f) O^T += U^T P^T      M=128 N=64  K=64
//   (g) S   += U^T Kt       M=128 N=128 K=64    (state update, fp32 in TMEM)
// Operands are fp16 tiles in 128-byte-swizzled shared memory (bf16 inputs are
// converted exactly on load; fp16 carries 3 more mantissa bits than bf16 at the
// same tensor-core rate, which keeps the bf16-output error at one rounding step;
// values must stay inside the fp16 range, |x| < 65504, which the recurrence with
// normalised keys does by a wide margin — an overflow shows up as inf/NaN); the
// fp32 state never leaves TMEM between chunks (its bf16 copy in shared memory is
// the operand of (d)/(e)).  The 64x64 triangular inverse is a blocked forward
// substitution in fp32 on the CUDA cores.  One CTA per (batch, head).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include "common.cuh"
#include "tc05.cuh"

namespace fo {
int gdr_stepwise(const void* q, const void* k, const void* v, const void* beta, const void* g,
                 const float* h0, void* o, float* hT, int64_t B, int64_t H, int64_t L, int64_t D,
                 int dtype, int gate_dtype, cudaStream_t st, const int* only = nullptr);

__device__ unsigned int g_gdr_timeouts;

namespace {

constexpr int kC = 64;
constexpr int kD = 128;
constexpr int kThr = 256;
constexpr uint32_t kWaitLimit = 1u << 22;

// shared-memory map (bytes from a 1024-aligned base).  Owner: P = prep warps,
// C = chain warps, P->C = written by prep, read by the chain (single buffer,
// guarded by the chain's MMA-completion barriers).
constexpr uint32_t OFF_QK = 0;         // P    2 x [128 x 128B]: rows 0-63 Q, 64-127 K (then gK)  tile set 0
constexpr uint32_t OFF_V = 32768;      // P    2 x [64 x 128B]   V                               tile set 0
constexpr uint32_t OFF_GQ = 49152;     // P->C 2 x [64 x 128B]   gQ
constexpr uint32_t OFF_KT = 65536;     // P->C 2 x [64 x 128B]   Kt
constexpr uint32_t OFF_WT = 81920;     // P->C [128 x 128B]      -W^T
constexpr uint32_t OFF_P = 98304;      // C    [64 x 128B]       P
constexpr uint32_t OFF_S = 106496;     // C    2 x [128 x 128B]  state (fp16 copy)
constexpr uint32_t OFF_UT = 139264;    // C    [128 x 128B]      U^T; then output staging [64 x 256B]
constexpr uint32_t OFF_SET1 = 155648;  // P    tile set 1: QK at +0, V at +32768 (48 KB)
constexpr uint32_t OFF_T = 204800;     // P    2 x [64 x 128B]   T = (I + A)^-1 (gdr_tinv_kernel)
constexpr uint32_t OFF_G = 222208;     // gate tables x 2 (P->C), then barriers
constexpr int kAStride = 68;
constexpr uint32_t kGateBytes = 2304;
constexpr uint32_t G_LC = 0, G_Z = 256, G_NEG = 512, G_BETA = 768, G_GAM = 1024, G_GAMP = 1280,
                   G_KTS = 1536, G_SB = 1792, G_GC = 2048;
constexpr uint32_t OFF_BAR = OFF_G + 2 * kGateBytes;
constexpr uint32_t kSmemBytes = OFF_BAR + 128 + 1024;  // + alignment slack

// TMEM columns (fp32 accumulators, 128 lanes): chain-owned S, O; double-buffered
// U (prep writes U0, chain accumulates and reads) and QK^T/KK^T; prep-owned W.
constexpr uint32_t TM_S = 0, TM_O = 128, TM_U0 = 192, TM_QK0 = 320, TM_W = 448, TM_COLS = 512;

// element type of every tensor-core operand tile
using Op = __half;

// 8 input elements (16 bytes of T) -> 8 fp16 operand elements
template <typename T>
__device__ __forceinline__ uint4 to_op8(uint4 u) {
  if constexpr (std::is_same<T, __half>::value) {
    return u;
  } else {
    // a bf16 pair in one word: low half << 16 and high half & 0xffff0000 are its floats
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 h = __floats2half2_rn(__uint_as_float(w[i] << 16),
                                          __uint_as_float(w[i] & 0xffff0000u));
      w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return u;
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (std::is_same<T, __half>::value) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

// packed fp32x2 arithmetic (one instruction for two lanes of a float2)
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(r)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)),
        "l"(*reinterpret_cast<uint64_t*>(&c)));
  return *reinterpret_cast<float2*>(&r);
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;"
      : "=l"(r)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)));
  return *reinterpret_cast<float2*>(&r);
}

// 8 fp16 values times a scale (HMUL2; the product is rounded to fp16 as the
// operand tile would be anyway)
__device__ __forceinline__ uint4 scale8h(uint4 u, __half2 s) {
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __hmul2(h[i], s);
  return u;
}

// 8 input elements times a scale, as fp16 operand elements: fp16 input in
// half2 arithmetic (as above); bf16 input unpacked, scaled in fp32 and rounded
// once to fp16
template <typename T>
__device__ __forceinline__ uint4 scale8_op(uint4 u, float s) {
  if constexpr (std::is_same<T, __half>::value) {
    return scale8h(u, __float2half2_rn(s));
  } else {
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 h = __floats2half2_rn(__uint_as_float(w[i] << 16) * s,
                                          __uint_as_float(w[i] & 0xffff0000u) * s);
      w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return u;
  }
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// lc: in-chunk prefix sums of log2|g|; z: last zero-gate index (-1 if none);
// neg: prefix count of negative gates.
struct GateTabs {
  const float* lc;
  const int* z;
  const int* neg;
  // ratio(t, s) = gamma_t / gamma_s for -1 <= s <= t
  __device__ __forceinline__ float ratio(int t, int s) const {
    if (s >= t) return 1.f;
    if (z[t] > s) return 0.f;
    const float e = lc[t] - (s >= 0 ? lc[s] : 0.f);
    const int par = (neg[t] - (s >= 0 ? neg[s] : 0)) & 1;
    const float r = exp2f(e);
    return par ? -r : r;
  }
};

template <typename T, typename G>
__global__ void __launch_bounds__(kThr, 1)
gdr_tc_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
              const G* __restrict__ beta, const G* __restrict__ g, const float* __restrict__ h0,
              T* __restrict__ o, float* __restrict__ hT, int* __restrict__ flags,
              const __half* __restrict__ tin, const __grid_constant__ CUtensorMap tmq,
              const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
              int64_t L, int D) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~(uintptr_t)1023);
  const uint32_t sb = tc::smem_u32(sm);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  // bars[0], bars[7]: tile set 0 / 1 loaded (prep)
  uint64_t* bar_pmma = bars + 1;   // prep's MMAs completed                  (prep)
  uint64_t* bar_prep = bars + 2;   // prep products of a chunk ready         (prep -> chain)
  uint64_t* bar_b1 = bars + 3;     // chain MMAs (d),(e) completed           (chain -> both)
  uint64_t* bar_b2 = bars + 4;     // chain MMAs (f),(g) completed           (chain -> both)
  uint64_t* bar_done = bars + 5;   // [2] chain finished a chunk (per buffer) (chain -> prep)
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 64);
  int* s_abort = reinterpret_cast<int*>(sm + OFF_BAR + 68);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool is_chain = warp < 4;
  const int gt_id = is_chain ? tid : tid - 128;   // thread index inside its group
  const int quad = warp & 3;                      // TMEM lane quadrant
  const int row = 32 * quad + lane;               // TMEM lane = accumulator row
  const int64_t head = blockIdx.x;
  // a head dimension D < 128 runs as D = 128 with zero channels: the tensor
  // maps fill the columns past D with zeros, which leave every product, the
  // outputs' first D channels and the state's D x D block exact
  T* oh = o + head * L * D;
  const G* bh = beta + head * L;
  const G* gh = g + head * L;
  constexpr bool BF = false;  // operands are fp16 (except MMA (a): the input type)
  constexpr bool kInBF = std::is_same<T, __nv_bfloat16>::value;
  const int64_t nchunks = (L + kC - 1) / kC;
  const int bar_id = is_chain ? 1 : 2;            // named barrier of the group

  if (warp == 0) {
    tc::tmem_alloc(s_tmem, TM_COLS);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int b = 0; b < 8; ++b) tc::mbar_init(bars + b, 1);
    tc::fence_mbar_init();
    *s_abort = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tm = *s_tmem;
  const uint32_t tm_lane = tm + ((uint32_t)(32 * quad) << 16);

  auto gsync = [&]() {
    tc::fence_before_sync();
    asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
    tc::fence_after_sync();
  };
  // One elected thread of the group polls the mbarrier (bounded); a reducing
  // group barrier hands every thread of the group the same abort decision, so a
  // timeout (or the other group giving up) can never split a group across a
  // barrier.  Returns true when the group must stop.
  auto gwait = [&](uint64_t* bar, uint32_t parity) -> bool {
    int bad = 0;
    if (gt_id == 0) {
      if (*reinterpret_cast<volatile int*>(s_abort)) {
        bad = 1;
      } else if (!tc::mbar_wait(bar, parity, kWaitLimit)) {
        atomicAdd(&g_gdr_timeouts, 1u);
        *reinterpret_cast<volatile int*>(s_abort) = 1;
        bad = 1;
      }
    }
    tc::fence_before_sync();
    int any;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.s32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, 128, p;\n\t"
        "selp.s32 %0, 1, 0, q;\n\t}"
        : "=r"(any)
        : "r"(bad), "r"(bar_id)
        : "memory");
    tc::fence_after_sync();
    return any != 0;
  };
  auto gtab = [&](int b) { return sm + OFF_G + b * kGateBytes; };
  // fp16 range guard.  An operand that leaves the fp16 range becomes inf, and
  // an inf reaches every later output through the products (as inf or NaN,
  // 0 * inf included), so the chain group watches what it writes: the fp32
  // outputs o and the final state.  nf = sum of 0 * x stays 0 while every x is
  // finite and turns NaN at the first non-finite one (one FMA per value).
  float nf = 0.f;

  if (!is_chain) {
    // =====================================================================
    // prep warps: everything of a chunk that does not need the state
    // =====================================================================
    const int p = gt_id;
    uint32_t pmma_phase = 0;
    // Chunk c's q, k, v tiles land by TMA (bf16/fp16, 128-byte swizzled, rows
    // past the head's end zero-filled) in tile set c & 1, together with its T
    // tile; chunk c + 1's loads are issued when chunk c starts, so they have a
    // whole chunk to arrive.
    static_assert(OFF_V == OFF_QK + 32768, "a tile set is QK then V");
    auto set_base = [&](int64_t c) -> uint32_t { return (c & 1) ? OFF_SET1 : OFF_QK; };
    auto ld_bar = [&](int64_t c) -> uint64_t* { return (c & 1) ? bars + 7 : bars + 0; };
    int64_t issued = -1, landed = -1;
    auto issue_load = [&](int64_t c) {
      const uint32_t base = set_base(c);
      uint64_t* bar = ld_bar(c);
      tc::mbar_arrive_expect_tx(bar, 6 * 8192 + 8192);
      const int t0 = (int)(c * kC), hz = (int)head;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        tc::tma_load_3d(sm + base + h * 16384, &tmq, 64 * h, t0, hz, bar);
        tc::tma_load_3d(sm + base + h * 16384 + 8192, &tmk, 64 * h, t0, hz, bar);
        tc::tma_load_3d(sm + base + 32768 + h * 8192, &tmv, 64 * h, t0, hz, bar);
      }
      // T = (I + A)^-1 of the chunk, made by gdr_tinv_kernel, into T buffer c & 1
      tc::bulk_g2s(sm + OFF_T + (uint32_t)(c & 1) * 8192, tin + (head * nchunks + c) * (kC * 64),
                   8192, bar);
    };
    auto pmma_wait = [&]() -> bool {
      const bool bad = gwait(bar_pmma, pmma_phase);
      pmma_phase ^= 1u;
      return bad;
    };
    if (p == 0 && nchunks > 0) issue_load(0);
    issued = 0;
    float nb_gate = 0.f, ng_gate = 1.f;
    if (p < 64 && p < L) {
      nb_gate = to_f<G>(bh[p]);
      ng_gate = to_f<G>(gh[p]);
    }
    for (int64_t c = 0; c < nchunks; ++c) {
      const int b = (int)(c & 1);
      const int64_t tok0 = c * kC;
      const uint32_t QKs = set_base(c), Vs = QKs + 32768;
      uint8_t* G0 = gtab(b);
      float* sLc = reinterpret_cast<float*>(G0 + G_LC);
      int* sZ = reinterpret_cast<int*>(G0 + G_Z);
      int* sNeg = reinterpret_cast<int*>(G0 + G_NEG);
      float* sBeta = reinterpret_cast<float*>(G0 + G_BETA);
      const GateTabs gt{sLc, sZ, sNeg};
      // buffers QK[b], U[b] and gate table b were last used by chunk c - 2
      if (c >= 2 && gwait(bar_done + b, (uint32_t)(((c - 2) >> 1) & 1))) break;
      // tile set (c + 1) & 1 and T buffer (c + 1) & 1 were last read by chunk
      // c - 1, whose MMAs and scaled copies are complete
      if (p == 0 && c + 1 < nchunks) issue_load(c + 1);
      if (c + 1 < nchunks) issued = c + 1;
      if (p < 64) {
        const float bt = nb_gate, gg = ng_gate;
        const int64_t t1 = tok0 + kC + p;
        nb_gate = t1 < L ? to_f<G>(bh[t1]) : 0.f;
        ng_gate = t1 < L ? to_f<G>(gh[t1]) : 1.f;
        sBeta[p] = bt;
        float lg = (gg != 0.f) ? log2f(fabsf(gg)) : 0.f;
        int zi = (gg == 0.f) ? p : -1;
        int ng = (gg < 0.f) ? 1 : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const float a = __shfl_up_sync(0xffffffffu, lg, off);
          const int bz = __shfl_up_sync(0xffffffffu, zi, off);
          const int bn = __shfl_up_sync(0xffffffffu, ng, off);
          if (lane >= off) {
            lg += a;
            zi = max(zi, bz);
            ng += bn;
          }
        }
        sLc[p] = lg;
        sZ[p] = zi;
        sNeg[p] = ng;
      }
      const bool ld_bad = gwait(ld_bar(c), (uint32_t)((c >> 1) & 1));
      if (ld_bad) break;
      landed = c;
      if (p >= 32 && p < 64) {
        sLc[p] += sLc[31];
        sZ[p] = max(sZ[p], sZ[31]);
        sNeg[p] += sNeg[31];
      }
      if constexpr (!std::is_same<T, __half>::value) {
        // bf16 -> fp16 in place over the V tile (16 KB; the swizzle does not
        // matter elementwise): 8 chunks of 16 bytes per thread, all in flight.
        // Q and K stay bf16: MMA (a) takes them as they landed, and the scaled
        // copies convert while they scale.
        uint4 val[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          val[u] = *reinterpret_cast<const uint4*>(sm + Vs + (uint32_t)(p + 128 * u) * 16);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          *reinterpret_cast<uint4*>(sm + Vs + (uint32_t)(p + 128 * u) * 16) = to_op8<T>(val[u]);
      }
      tc::fence_proxy_async();
      gsync();
      if (p < 64) {
        float* sGam = reinterpret_cast<float*>(G0 + G_GAM);
        float* sGamP = reinterpret_cast<float*>(G0 + G_GAMP);
        float* sKts = reinterpret_cast<float*>(G0 + G_KTS);
        float* sSB = reinterpret_cast<float*>(G0 + G_SB);
        sSB[p] = (sNeg[p] & 1) ? -sBeta[p] : sBeta[p];
        sGam[p] = gt.ratio(p, -1);
        sGamP[p] = p > 0 ? gt.ratio(p - 1, -1) : 1.f;
        sKts[p] = gt.ratio(kC - 1, p) * sBeta[p];
        if (p == 0) *reinterpret_cast<float*>(G0 + G_GC) = gt.ratio(kC - 1, -1);
      }
      // ---- (a) [Q;K] K^T -> QK[b], on the input tiles (bf16 x bf16 or fp16 x fp16)
      if (p == 0) {
        constexpr uint32_t id_a = tc::idesc_f16(128, 64, kInBF, false, false);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t h = ks >> 2, kk = ks & 3;
          const uint64_t da = tc::desc_sw128(sb + QKs + h * 16384 + kk * 32, 16, 1024);
          const uint64_t db = tc::desc_sw128(sb + QKs + h * 16384 + 8192 + kk * 32, 16, 1024);
          tc::mma_f16(tm + TM_QK0 + 64 * b, da, db, id_a, ks > 0);
        }
        tc::mma_commit(bar_pmma);
      }
      if (pmma_wait()) break;
      // gQ, Kt and gK overwrite chain inputs of chunk c - 1: wait for its last MMAs
      if (c >= 1) {
        if (gwait(bar_b2, (uint32_t)((c - 1) & 1))) break;
      } else {
        gsync();
      }
      {
        // ---- scaled copies: gQ -> GQ, Kt -> KT, gK in place; 8 loads in flight
        const float* sGam = reinterpret_cast<const float*>(G0 + G_GAM);
        const float* sGamP = reinterpret_cast<const float*>(G0 + G_GAMP);
        const float* sKts = reinterpret_cast<const float*>(G0 + G_KTS);
#pragma unroll
        for (int m = 0; m < 2; ++m) {  // m = 0: Q rows (0-63), m = 1: K rows (64-127)
          uint4 raw[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int rem = p + 128 * u, t = rem >> 4, ch = rem & 15;
            raw[u] = *reinterpret_cast<const uint4*>(sm + QKs + (ch >> 3) * 16384 +
                                                     tc::sw128_chunk(64 * m + t, ch & 7));
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int rem = p + 128 * u, t = rem >> 4, ch = rem & 15;
            const int half = ch >> 3, cc = ch & 7;
            if (m == 0) {
              *reinterpret_cast<uint4*>(sm + OFF_GQ + half * 8192 + tc::sw128_chunk(t, cc)) =
                  scale8_op<T>(raw[u], sGam[t]);
            } else {
              *reinterpret_cast<uint4*>(sm + OFF_KT + half * 8192 + tc::sw128_chunk(t, cc)) =
                  scale8_op<T>(raw[u], sKts[t]);
              *reinterpret_cast<uint4*>(sm + QKs + half * 16384 + tc::sw128_chunk(64 + t, cc)) =
                  scale8_op<T>(raw[u], sGamP[t]);
            }
          }
        }
      }
      tc::fence_proxy_async();
      gsync();
      // ---- (b) W^T = (gK)^T T^T -> W,  (c) U0^T = V^T T^T -> U[b]
      if (p == 0) {
        constexpr uint32_t id_mn = tc::idesc_f16(128, 64, BF, true, false);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t dt = tc::desc_sw128(sb + OFF_T + (uint32_t)b * 8192 + ks * 32, 16, 1024);
          const uint64_t dk = tc::desc_sw128(sb + QKs + 8192 + ks * 2048, 16384, 1024);
          const uint64_t dv = tc::desc_sw128(sb + Vs + ks * 2048, 8192, 1024);
          tc::mma_f16(tm + TM_W, dk, dt, id_mn, ks > 0);
          tc::mma_f16(tm + TM_U0 + 64 * b, dv, dt, id_mn, ks > 0);
        }
        tc::mma_commit(bar_pmma);
      }
      if (pmma_wait()) break;
      // ---- -W^T -> fp16 tile [j][t] (overwrites T, consumed by (b),(c))
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t r[32];
        tc::tmem_ld32(tm_lane + TM_W + 32 * hf, r);
        tc::tmem_wait_ld();
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint4 pk;
          pk.x = pack2<Op>(-__uint_as_float(r[8 * c4 + 0]), -__uint_as_float(r[8 * c4 + 1]));
          pk.y = pack2<Op>(-__uint_as_float(r[8 * c4 + 2]), -__uint_as_float(r[8 * c4 + 3]));
          pk.z = pack2<Op>(-__uint_as_float(r[8 * c4 + 4]), -__uint_as_float(r[8 * c4 + 5]));
          pk.w = pack2<Op>(-__uint_as_float(r[8 * c4 + 6]), -__uint_as_float(r[8 * c4 + 7]));
          *reinterpret_cast<uint4*>(sm + OFF_WT + tc::sw128_chunk(row, 4 * hf + c4)) = pk;
        }
      }
      tc::fence_proxy_async();
      gsync();
      if (p == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar_prep))
                               : "memory");
    }
    // an abort can leave tile loads in flight: let them land before exiting
    if (*s_abort && p == 0)
      for (int64_t c = landed + 1; c <= issued; ++c)
        tc::mbar_wait(ld_bar(c), (uint32_t)((c >> 1) & 1), kWaitLimit);
  } else {
    // =====================================================================
    // chain warps: the state-dependent part of each chunk
    // =====================================================================
    const int i = row;  // state row / value channel
    bool state_nz = false;
    if (h0) {
      const float* hh = h0 + head * D * D;
#pragma unroll
      for (int hq = 0; hq < 4; ++hq) {
        const int j0 = 32 * hq;
        uint32_t r[32];
#pragma unroll
        for (int j = 0; j < 32; ++j)
          r[j] = (i < D && j0 + j < D) ? __float_as_uint(hh[i * D + j0 + j]) : 0u;
        tc::tmem_st32(tm_lane + TM_S + j0, r);
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint4 pk;
          pk.x = pack2<Op>(__uint_as_float(r[8 * c4 + 0]), __uint_as_float(r[8 * c4 + 1]));
          pk.y = pack2<Op>(__uint_as_float(r[8 * c4 + 2]), __uint_as_float(r[8 * c4 + 3]));
          pk.z = pack2<Op>(__uint_as_float(r[8 * c4 + 4]), __uint_as_float(r[8 * c4 + 5]));
          pk.w = pack2<Op>(__uint_as_float(r[8 * c4 + 6]), __uint_as_float(r[8 * c4 + 7]));
          *reinterpret_cast<uint4*>(sm + OFF_S + (hq >> 1) * 16384 +
                                    tc::sw128_chunk(i, 4 * (hq & 1) + c4)) = pk;
        }
      }
      tc::tmem_wait_st();
      tc::fence_proxy_async();
      state_nz = true;
    }
    // The state in TMEM enters chunk c already multiplied by gamma_{C-1} of
    // chunk c (the previous chunk's state copy applies it), so (g) accumulates
    // onto it directly; (d),(e) read the undecayed fp16 copy.
    bool prep_ready = false;  // bar_prep of this chunk already waited for
    for (int64_t c = 0; c < nchunks; ++c) {
      const int b = (int)(c & 1);
      const uint32_t ph = (uint32_t)(c & 1);
      const int64_t tok0 = c * kC;
      const int nvalid = (int)((L - tok0) < kC ? (L - tok0) : kC);
      const uint8_t* G0 = gtab(b);
      const float* sLc = reinterpret_cast<const float*>(G0 + G_LC);
      const int* sZ = reinterpret_cast<const int*>(G0 + G_Z);
      const int* sNeg = reinterpret_cast<const int*>(G0 + G_NEG);
      const float* sSB = reinterpret_cast<const float*>(G0 + G_SB);
      if (!prep_ready && gwait(bar_prep, ph)) break;
      prep_ready = false;
      // ---- (d) U^T[b] += S (-W)^T,  (e) O^T = S (gQ)^T   (need the state)
      if (gt_id == 0) {
        if (state_nz) {
          constexpr uint32_t id_d = tc::idesc_f16(128, 64, BF, false, true);
          constexpr uint32_t id_e = tc::idesc_f16(128, 64, BF, false, false);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint32_t h = ks >> 2, kk = ks & 3;
            const uint64_t ds = tc::desc_sw128(sb + OFF_S + h * 16384 + kk * 32, 16, 1024);
            const uint64_t dw = tc::desc_sw128(sb + OFF_WT + ks * 2048, 8192, 1024);
            const uint64_t dq = tc::desc_sw128(sb + OFF_GQ + h * 8192 + kk * 32, 16, 1024);
            tc::mma_f16(tm + TM_U0 + 64 * b, ds, dw, id_d, 1);
            tc::mma_f16(tm + TM_O, ds, dq, id_e, ks > 0);
          }
          tc::mma_commit(bar_b1);
        } else {
          asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar_b1))
                       : "memory");
        }
      }
      // ---- P (rows 0-63 of QK[b]) while (d),(e) run: P[t][s] = ratio(t,s) beta_s (q_t . k_s)
      if (quad < 2) {
        const int t = row;
        const float lt = sLc[t];
        const int zr = sZ[t];
        const float sg = (sNeg[t] & 1) ? -1.f : 1.f;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t r[32];
          tc::tmem_ld32(tm_lane + TM_QK0 + 64 * b + 32 * hf, r);
          tc::tmem_wait_ld();
          float pv[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int s = 32 * hf + j;
            const bool on = (s <= t) && (zr <= s);
            pv[j] = on ? sg * sSB[s] * ex2(lt - sLc[s]) * __uint_as_float(r[j]) : 0.f;
          }
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            uint4 pk;
            pk.x = pack2<Op>(pv[8 * c4 + 0], pv[8 * c4 + 1]);
            pk.y = pack2<Op>(pv[8 * c4 + 2], pv[8 * c4 + 3]);
            pk.z = pack2<Op>(pv[8 * c4 + 4], pv[8 * c4 + 5]);
            pk.w = pack2<Op>(pv[8 * c4 + 6], pv[8 * c4 + 7]);
            *reinterpret_cast<uint4*>(sm + OFF_P + tc::sw128_chunk(t, 4 * hf + c4)) = pk;
          }
        }
      }
      tc::fence_proxy_async();
      if (gwait(bar_b1, ph)) break;
      // ---- U^T -> fp16 tile [i][s]; decay the fp32 state by gamma_{C-1}
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t r[32];
        tc::tmem_ld32(tm_lane + TM_U0 + 64 * b + 32 * hf, r);
        tc::tmem_wait_ld();
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint4 pk;
          pk.x = pack2<Op>(__uint_as_float(r[8 * c4 + 0]), __uint_as_float(r[8 * c4 + 1]));
          pk.y = pack2<Op>(__uint_as_float(r[8 * c4 + 2]), __uint_as_float(r[8 * c4 + 3]));
          pk.z = pack2<Op>(__uint_as_float(r[8 * c4 + 4]), __uint_as_float(r[8 * c4 + 5]));
          pk.w = pack2<Op>(__uint_as_float(r[8 * c4 + 6]), __uint_as_float(r[8 * c4 + 7]));
          *reinterpret_cast<uint4*>(sm + OFF_UT + tc::sw128_chunk(i, 4 * hf + c4)) = pk;
        }
      }
      if (state_nz && c == 0) {
        // the initial state: decayed here (later chunks' by the state copy)
        const float gc = *reinterpret_cast<const float*>(G0 + G_GC);
#pragma unroll
        for (int hq = 0; hq < 4; ++hq) {
          uint32_t r[32];
          tc::tmem_ld32(tm_lane + TM_S + 32 * hq, r);
          tc::tmem_wait_ld();
          const float2 g2 = make_float2(gc, gc);
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float2 m2 = mul2(make_float2(__uint_as_float(r[j]), __uint_as_float(r[j + 1])), g2);
            r[j] = __float_as_uint(m2.x);
            r[j + 1] = __float_as_uint(m2.y);
          }
          tc::tmem_st32(tm_lane + TM_S + 32 * hq, r);
        }
        tc::tmem_wait_st();
      }
      tc::fence_proxy_async();
      gsync();
      // ---- (f) O^T += U^T P^T,  (g) S (+)= U^T Kt
      if (gt_id == 0) {
        constexpr uint32_t id_f = tc::idesc_f16(128, 64, BF, false, false);
        constexpr uint32_t id_g = tc::idesc_f16(128, 128, BF, false, true);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t du = tc::desc_sw128(sb + OFF_UT + ks * 32, 16, 1024);
          const uint64_t dp = tc::desc_sw128(sb + OFF_P + ks * 32, 16, 1024);
          const uint64_t dk = tc::desc_sw128(sb + OFF_KT + ks * 2048, 8192, 1024);
          tc::mma_f16(tm + TM_O, du, dp, id_f, (state_nz || ks > 0) ? 1u : 0u);
          tc::mma_f16(tm + TM_S, du, dk, id_g, (state_nz || ks > 0) ? 1u : 0u);
        }
        tc::mma_commit(bar_b2);
      }
      if (gwait(bar_b2, ph)) break;
      state_nz = true;
      // ---- O^T -> staging [t][i] (U^T buffer, consumed) -> global
      {
        uint32_t r[32];
        T* so = reinterpret_cast<T*>(sm + OFF_UT);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          tc::tmem_ld32(tm_lane + TM_O + 32 * hf, r);
          tc::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float x = __uint_as_float(r[j]);
            nf = fmaf(0.f, x, nf);
            so[(32 * hf + j) * kD + i] = from_f<T>(x);
          }
        }
      }
      gsync();
      const int nch = D >> 3;  // 16-byte chunks of an output row
      for (int e = gt_id; e < nvalid * nch; e += 128) {
        const int t = e / nch, ch = e - t * nch;
        st_global_v4(oh + (tok0 + t) * D + ch * 8,
                     *reinterpret_cast<const uint4*>(sm + OFF_UT + t * 256 + ch * 16));
      }
      gsync();  // staging read before the next chunk's U^T overwrites it
      if (gt_id == 0)
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar_done + b))
                     : "memory");
      // ---- the state for chunk c + 1: its fp16 operand copy (undecayed, for
      // (d),(e)), and the TMEM state multiplied by chunk c + 1's gamma_{C-1}
      // (what (g) accumulates onto), in one pass over the state
      if (c + 1 < nchunks) {
        if (gwait(bar_prep, ph ^ 1u)) break;  // chunk c + 1's gate table is ready
        prep_ready = true;
        const float gn = *reinterpret_cast<const float*>(gtab(b ^ 1) + G_GC);
        const float2 g2 = make_float2(gn, gn);
        uint32_t r[32];
#pragma unroll
        for (int hq = 0; hq < 4; ++hq) {
          tc::tmem_ld32(tm_lane + TM_S + 32 * hq, r);
          tc::tmem_wait_ld();
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            uint4 pk;
            pk.x = pack2<Op>(__uint_as_float(r[8 * c4 + 0]), __uint_as_float(r[8 * c4 + 1]));
            pk.y = pack2<Op>(__uint_as_float(r[8 * c4 + 2]), __uint_as_float(r[8 * c4 + 3]));
            pk.z = pack2<Op>(__uint_as_float(r[8 * c4 + 4]), __uint_as_float(r[8 * c4 + 5]));
            pk.w = pack2<Op>(__uint_as_float(r[8 * c4 + 6]), __uint_as_float(r[8 * c4 + 7]));
            *reinterpret_cast<uint4*>(sm + OFF_S + (hq >> 1) * 16384 +
                                      tc::sw128_chunk(i, 4 * (hq & 1) + c4)) = pk;
          }
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float2 m2 = mul2(make_float2(__uint_as_float(r[j]), __uint_as_float(r[j + 1])), g2);
            r[j] = __float_as_uint(m2.x);
            r[j + 1] = __float_as_uint(m2.y);
          }
          tc::tmem_st32(tm_lane + TM_S + 32 * hq, r);
        }
        tc::tmem_wait_st();
        tc::fence_proxy_async();
        gsync();
      }
    }
    // ---- final state
    if (hT && !*s_abort) {
      float* hh = hT + head * D * D;
#pragma unroll
      for (int hq = 0; hq < 4; ++hq) {
        uint32_t r[32];
        if (state_nz) {
          tc::tmem_ld32(tm_lane + TM_S + 32 * hq, r);
          tc::tmem_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = 0u;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) nf = fmaf(0.f, __uint_as_float(r[j]), nf);
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4)
          if (i < D && 32 * hq + 4 * j4 < D)
            *reinterpret_cast<uint4*>(hh + i * D + 32 * hq + 4 * j4) =
                make_uint4(r[4 * j4], r[4 * j4 + 1], r[4 * j4 + 2], r[4 * j4 + 3]);
      }
    }
  }
  // a head with a non-finite output (an fp16 operand overflowed, or the inputs
  // were not finite) or that gave up on a wait is marked for recomputation by
  // the fp32 per-step kernel
  const int bad = (nf != nf) || *reinterpret_cast<volatile int*>(s_abort);
  tc::fence_before_sync();
  const int any_bad = __syncthreads_or(bad);
  if (tid == 0 && flags) flags[head] = any_bad;
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tm, TM_COLS);
  }
}

// ---------------------------------------------------------------------------
// T = (I + A)^-1 of every (head, chunk): the one step of a chunk's preparation
// with a long dependency chain (the triangular solve), run for all chunks in
// parallel before the scan kernel, with several CTAs per SM hiding each
// other's latency.  Output: per (head, chunk) the fp16 T tile [t][s] in the
// 128-byte-swizzled layout the scan kernel's MMAs read (8 KB), copied there
// as it is.
// ---------------------------------------------------------------------------
constexpr int kTiThr = 128;
constexpr uint32_t TI_K = 0;         // fp16 2 x [128 x 128B]: rows 0-63 K, rows 64-127 K again,
                                     // so K K^T lands in all four TMEM lane quadrants
constexpr uint32_t TI_OUT = 32768;   // fp16 T tile [64 x 128B]
constexpr uint32_t TI_A = 40960;     // fp32 [64][68]: N = -A stored transposed
constexpr uint32_t TI_TSC = 58368;   // fp32 [64][kTscStride]: T00 (rows 0-31) | T11 (rows 32-63)
constexpr int kTscStride = 36;       // 144-byte rows: 16-byte aligned, and the 8 rows a warp reads
                                     // in T10 = T11 P start on 8 different banks
constexpr uint32_t TI_G = 67584;     // lc, z, neg, signed beta: 64 each
constexpr uint32_t TI_BAR = 68608;   // mbarrier, TMEM address
constexpr uint32_t kTiSmem = TI_BAR + 64 + 1024;  // + alignment slack
constexpr uint32_t kTiCols = 64;

template <typename T, typename G>
__global__ void __launch_bounds__(kTiThr, 3)
gdr_tinv_kernel(const T* __restrict__ k, const G* __restrict__ beta, const G* __restrict__ g,
                __half* __restrict__ tout, int64_t L, int64_t items, int D) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~(uintptr_t)1023);
  const uint32_t sb = tc::smem_u32(sm);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + TI_BAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + TI_BAR + 16);
  float* sA = reinterpret_cast<float*>(sm + TI_A);
  float* Tsc = reinterpret_cast<float*>(sm + TI_TSC);
  float* sLc = reinterpret_cast<float*>(sm + TI_G);
  int* sZ = reinterpret_cast<int*>(sm + TI_G + 256);
  int* sNeg = reinterpret_cast<int*>(sm + TI_G + 512);
  float* sSB = reinterpret_cast<float*>(sm + TI_G + 768);
  const int p = threadIdx.x, lane = p & 31, warp = p >> 5;
  const int64_t nchunks = (L + kC - 1) / kC;
  if (warp == 0) {
    tc::tmem_alloc(s_tmem, kTiCols);
    tc::tmem_relinquish();
  }
  if (p == 0) {
    tc::mbar_init(bar, 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tm = *s_tmem;
  const uint32_t tm_lane = tm + ((uint32_t)(32 * (warp & 3)) << 16);
  uint32_t phase = 0;

  // the k rows of an item: chunk j = p + 128 u of the 1024 16-byte chunks
  uint4 val[8];
  float bt = 0.f, gg = 1.f;
  auto fetch = [&](int64_t it) {
    if (it >= items) return;
    const int64_t head = it / nchunks, c = it % nchunks;
    const int64_t t0 = c * kC;
    const int nvalid = (int)((L - t0) < kC ? (L - t0) : kC);
    const T* kr = k + (head * L + t0) * D;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      // channels past D (D < 128) are zeros
      const int idx = p + 128 * u, t = idx >> 4, ch = idx & 15;
      val[u] = (t < nvalid && ch * 8 < D) ? ld_global_stream_v4(kr + t * D + ch * 8)
                                           : make_uint4(0, 0, 0, 0);
    }
    if (p < 64) {
      bt = p < nvalid ? to_f<G>(beta[head * L + t0 + p]) : 0.f;
      gg = p < nvalid ? to_f<G>(g[head * L + t0 + p]) : 1.f;
    }
  };
  fetch(blockIdx.x);
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    // ---- fp16 K tile and gate tables
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int idx = p + 128 * u, t = idx >> 4, ch = idx & 15;
      const uint4 h = to_op8<T>(val[u]);
      *reinterpret_cast<uint4*>(sm + TI_K + (ch >> 3) * 16384 + tc::sw128_chunk(t, ch & 7)) = h;
      *reinterpret_cast<uint4*>(sm + TI_K + (ch >> 3) * 16384 + tc::sw128_chunk(64 + t, ch & 7)) =
          h;
    }
    if (p < 64) {
      float lg = (gg != 0.f) ? log2f(fabsf(gg)) : 0.f;
      int zi = (gg == 0.f) ? p : -1;
      int ng = (gg < 0.f) ? 1 : 0;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float a = __shfl_up_sync(0xffffffffu, lg, off);
        const int bz = __shfl_up_sync(0xffffffffu, zi, off);
        const int bn = __shfl_up_sync(0xffffffffu, ng, off);
        if (lane >= off) {
          lg += a;
          zi = max(zi, bz);
          ng += bn;
        }
      }
      sLc[p] = lg;
      sZ[p] = zi;
      sNeg[p] = ng;
      sSB[p] = bt;
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (p >= 32 && p < 64) {
      sLc[p] += sLc[31];
      sZ[p] = max(sZ[p], sZ[31]);
      sNeg[p] += sNeg[31];
    }
    // ---- K K^T (TMEM lanes 0-63)
    if (p == 0) {
      constexpr uint32_t id = tc::idesc_f16(128, 64, false, false, false);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t h = ks >> 2, kk = ks & 3;
        const uint64_t d = tc::desc_sw128(sb + TI_K + h * 16384 + kk * 32, 16, 1024);
        tc::mma_f16(tm, d, d, id, ks > 0);  // A: all 128 rows; B: rows 0-63
      }
      tc::mma_commit(bar);
    }
    fetch(it + gridDim.x);  // the next item's loads fly during this one
    __syncthreads();
    if (p < 64) sSB[p] = (sNeg[p] & 1) ? -sSB[p] : sSB[p];
    int good = 1;
    if (p == 0) good = tc::mbar_wait(bar, phase, kWaitLimit) ? 1 : 0;  // one poller
    phase ^= 1u;
    if (!__syncthreads_and(good)) {
      if (p == 0) atomicAdd(&g_gdr_timeouts, 1u);
      break;
    }
    tc::fence_after_sync();
    // ---- N = -A, stored transposed: sA[s][t] = -ratio(t-1,s) beta_s (k_t . k_s), s < t
    {
      // warps 0, 1: rows 0-63 (lanes 0-63), columns 0-31; warps 2, 3: the same
      // rows from the copy in lanes 64-127, columns 32-63
      const int t = 32 * (warp & 1) + lane, tr = t - 1, hf = warp >> 1;
      const float lt = tr >= 0 ? sLc[tr] : 0.f;
      const int zr = tr >= 0 ? sZ[tr] : -1;
      const float sg = (tr >= 0 && (sNeg[tr] & 1)) ? -1.f : 1.f;
      {
        uint32_t r[32];
        tc::tmem_ld32(tm_lane + 32 * hf, r);
        tc::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int s = 32 * hf + j;
          const bool on = (s <= tr) && (zr <= s);
          sA[s * kAStride + t] = on ? -sg * sSB[s] * ex2(lt - sLc[s]) * __uint_as_float(r[j]) : 0.f;
        }
      }
    }
    tc::fence_before_sync();
    __syncthreads();
    // ---- diagonal 32x32 blocks of T = (I - N)^-1, column by column (right-looking)
    if (p < 64) {
      const int I = p >> 5, cc = p & 31;
      const float* nb = sA + (32 * I) * kAStride + 32 * I;  // nb[i][a] = N[32I+a][32I+i]
      float2 col[16];
#pragma unroll
      for (int r = 0; r < 16; ++r)
        col[r] = make_float2((2 * r == cc) ? 1.f : 0.f, (2 * r + 1 == cc) ? 1.f : 0.f);
#pragma unroll
      for (int i = 0; i < 31; ++i) {
        const float ti = (i & 1) ? col[i / 2].y : col[i / 2].x;
        const float2 t2 = make_float2(ti, ti);
        const float* nc = nb + i * kAStride;
        int r = i + 1;
        if (r & 1) {
          col[r / 2].y = fmaf(nc[r], ti, col[r / 2].y);
          ++r;
        }
        if ((r & 3) && r < 32) {
          const float2 a2 = *reinterpret_cast<const float2*>(nc + r);
          col[r / 2] = fma2(a2, t2, col[r / 2]);
          r += 2;
        }
#pragma unroll
        for (; r < 32; r += 4) {
          const float4 a4 = *reinterpret_cast<const float4*>(nc + r);
          col[r / 2] = fma2(make_float2(a4.x, a4.y), t2, col[r / 2]);
          col[r / 2 + 1] = fma2(make_float2(a4.z, a4.w), t2, col[r / 2 + 1]);
        }
      }
#pragma unroll
      for (int a = 0; a < 32; ++a) {
        const float tv = (a & 1) ? col[a / 2].y : col[a / 2].x;
        Tsc[(32 * I + a) * kTscStride + cc] = tv;
        *reinterpret_cast<__half*>(sm + TI_OUT + tc::sw128_off(32 * I + a, p)) = __float2half_rn(tv);
        if (I == 1)
          *reinterpret_cast<__half*>(sm + TI_OUT + tc::sw128_off(a, p)) = __float2half_rn(0.f);
      }
    }
    __syncthreads();
    {
      // ---- P = N10 T00 -> sA[32 + a][b] (slots above the diagonal)
      const int a = p >> 2, b0 = (p & 3) * 8;
      float2 acc[4] = {};
#pragma unroll
      for (int d = 0; d < 32; ++d) {
        const float n = sA[d * kAStride + 32 + a];
        const float2 n2 = make_float2(n, n);
        const float4 t0 = *reinterpret_cast<const float4*>(Tsc + d * kTscStride + b0);
        const float4 t1 = *reinterpret_cast<const float4*>(Tsc + d * kTscStride + b0 + 4);
        acc[0] = fma2(n2, make_float2(t0.x, t0.y), acc[0]);
        acc[1] = fma2(n2, make_float2(t0.z, t0.w), acc[1]);
        acc[2] = fma2(n2, make_float2(t1.x, t1.y), acc[2]);
        acc[3] = fma2(n2, make_float2(t1.z, t1.w), acc[3]);
      }
      float* prow = sA + (32 + a) * kAStride + b0;
      *reinterpret_cast<float4*>(prow) = make_float4(acc[0].x, acc[0].y, acc[1].x, acc[1].y);
      *reinterpret_cast<float4*>(prow + 4) = make_float4(acc[2].x, acc[2].y, acc[3].x, acc[3].y);
    }
    __syncthreads();
    {
      // ---- T10 = T11 P -> rows 32-63, columns 0-31 of the T tile
      const int a = p >> 2, b0 = (p & 3) * 8;
      float2 acc[4] = {};
#pragma unroll
      for (int c2 = 0; c2 < 32; ++c2) {
        const float tv = Tsc[(32 + a) * kTscStride + c2];
        const float2 t2 = make_float2(tv, tv);
        const float4 p0 = *reinterpret_cast<const float4*>(sA + (32 + c2) * kAStride + b0);
        const float4 p1 = *reinterpret_cast<const float4*>(sA + (32 + c2) * kAStride + b0 + 4);
        acc[0] = fma2(t2, make_float2(p0.x, p0.y), acc[0]);
        acc[1] = fma2(t2, make_float2(p0.z, p0.w), acc[1]);
        acc[2] = fma2(t2, make_float2(p1.x, p1.y), acc[2]);
        acc[3] = fma2(t2, make_float2(p1.z, p1.w), acc[3]);
      }
      uint4 pk;
      pk.x = pack2<Op>(acc[0].x, acc[0].y);
      pk.y = pack2<Op>(acc[1].x, acc[1].y);
      pk.z = pack2<Op>(acc[2].x, acc[2].y);
      pk.w = pack2<Op>(acc[3].x, acc[3].y);
      *reinterpret_cast<uint4*>(sm + TI_OUT + tc::sw128_chunk(32 + a, b0 >> 3)) = pk;
    }
    __syncthreads();
    // ---- the 8 KB tile to global memory as it is
    {
      uint4* dst = reinterpret_cast<uint4*>(tout + it * (int64_t)(kC * 64));
      const uint4* srcv = reinterpret_cast<const uint4*>(sm + TI_OUT);
#pragma unroll
      for (int u = 0; u < 4; ++u) dst[p + 128 * u] = srcv[p + 128 * u];
    }
    __syncthreads();
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tm, kTiCols);
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point, so that the
// library has no link-time dependency on the driver library (it loads on
// machines without a GPU driver; the entry point is looked up on first use).
PFN_cuTensorMapEncodeTiled tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(p);
  }
  return fn;
}

template <typename T, typename G>
int launch_tc(const void* q, const void* k, const void* v, const void* beta, const void* g,
              const float* h0, void* o, float* hT, int* flags, __half* tbuf, int64_t BH,
              int64_t L, int D, cudaStream_t st) {
  // 1. T = (I + A)^-1 of every (head, chunk), all chunks in parallel
  auto tkern = gdr_tinv_kernel<T, G>;
  // several CTAs per SM hide each other's latency: ask for the largest shared
  // memory carve-out so that they fit
  if (cudaFuncSetAttribute(tkern, cudaFuncAttributeMaxDynamicSharedMemorySize, kTiSmem) !=
          cudaSuccess ||
      cudaFuncSetAttribute(tkern, cudaFuncAttributePreferredSharedMemoryCarveout,
                           (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess) {
    set_error("gdr_tinv_kernel: cannot reserve %u bytes of shared memory", kTiSmem);
    return FO_ECUDA;
  }
  // 3 CTAs per SM (shared memory and registers allow it); the CTAs never wait
  // on one another, so more of them than fit simply queue
  const int64_t items = BH * ((L + kC - 1) / kC);
  int64_t tgrid = (int64_t)num_sms() * 3;
  if (tgrid > items) tgrid = items;
  tkern<<<(unsigned)tgrid, kTiThr, kTiSmem, st>>>((const T*)k, (const G*)beta, (const G*)g, tbuf,
                                                  L, items, D);
  if (int rc = check_launch("gdr_tinv_kernel")) return rc;
  // 2. the chunk scan; q, k, v reach it through TMA tensor maps
  CUtensorMap maps[3];
  const void* srcs[3] = {q, k, v};
  // extent D in the channel dimension: for D < 128 the boxes past it (the
  // second 64-channel half, and channels D..63 of the first) are zero-filled
  const cuuint64_t gdim[3] = {(cuuint64_t)D, (cuuint64_t)L, (cuuint64_t)BH};
  const cuuint64_t gstride[2] = {(cuuint64_t)D * sizeof(T), (cuuint64_t)L * D * sizeof(T)};
  const cuuint32_t box[3] = {64, (cuuint32_t)kC, 1};
  const cuuint32_t estride[3] = {1, 1, 1};
  PFN_cuTensorMapEncodeTiled encode = tensor_map_encoder();
  if (!encode) {
    set_error("chunk_gated_delta_rule: the driver's cuTensorMapEncodeTiled is not available");
    return FO_ECUDA;
  }
  for (int i = 0; i < 3; ++i) {
    const CUresult r = encode(
        &maps[i], std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
        3, const_cast<void*>(srcs[i]), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("chunk_gated_delta_rule: cuTensorMapEncodeTiled failed (%d)", (int)r);
      return FO_ECUDA;
    }
  }
  auto kern = gdr_tc_kernel<T, G>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
      cudaSuccess) {
    set_error("gdr_tc_kernel: cannot reserve %u bytes of shared memory", kSmemBytes);
    return FO_ECUDA;
  }
  kern<<<(unsigned)BH, kThr, kSmemBytes, st>>>((const T*)q, (const T*)k, (const T*)v,
                                               (const G*)beta, (const G*)g, h0, (T*)o, hT, flags,
                                               tbuf, maps[0], maps[1], maps[2], L, D);
  return check_launch("gdr_tc_kernel");
}

template <typename T>
int tc_gate_dispatch(int gate_dtype, const void* q, const void* k, const void* v, const void* beta,
                     const void* g, const float* h0, void* o, float* hT, int* flags,
                     __half* tbuf, int64_t BH, int64_t L, int D, cudaStream_t st) {
  switch (gate_dtype) {
    case FO_F32:
      return launch_tc<T, float>(q, k, v, beta, g, h0, o, hT, flags, tbuf, BH, L, D, st);
    case FO_F16:
      return launch_tc<T, __half>(q, k, v, beta, g, h0, o, hT, flags, tbuf, BH, L, D, st);
    case FO_BF16:
      return launch_tc<T, __nv_bfloat16>(q, k, v, beta, g, h0, o, hT, flags, tbuf, BH, L, D, st);
  }
  set_error("chunk_gated_delta_rule: unsupported gate dtype code %d", gate_dtype);
  return FO_EDTYPE;
}

// ---------------------------------------------------------------------------
// operand-layout self-test: D[M=128, N] = A[128, K] B[N, K]^T, one CTA
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) tc_selftest_kernel(const __nv_bfloat16* __restrict__ a,
                                                          const __nv_bfloat16* __restrict__ b,
                                                          float* __restrict__ d, int N, int K,
                                                          int a_mn, int b_mn) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~(uintptr_t)1023);
  // A tile: K-major -> K/64 blocks of [128 rows x 128B]; MN-major -> 2 blocks of [K rows x 128B]
  // B tile: K-major -> K/64 blocks of [N rows x 128B];  MN-major -> N/64 blocks of [K rows x 128B]
  const uint32_t a_bytes = 128 * K * 2;
  uint8_t* sa = sm;
  uint8_t* sbm = sm + a_bytes;
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + a_bytes + N * K * 2);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(mbar + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // A logical element (m, kk)
  for (int e = tid; e < 128 * K; e += 128) {
    int m, kk;
    __nv_bfloat16 val;
    if (!a_mn) { m = e / K; kk = e % K; val = a[m * K + kk]; }
    else { kk = e / 128; m = e % 128; val = a[kk * 128 + m]; }
    uint32_t off;
    if (!a_mn) off = (kk / 64) * (128 * 128) + tc::sw128_off(m, kk % 64);
    else off = (m / 64) * (K * 128) + tc::sw128_off(kk, m % 64);
    *reinterpret_cast<__nv_bfloat16*>(sa + off) = val;
  }
  for (int e = tid; e < N * K; e += 128) {
    int n, kk;
    __nv_bfloat16 val;
    if (!b_mn) { n = e / K; kk = e % K; val = b[n * K + kk]; }
    else { kk = e / N; n = e % N; val = b[kk * N + n]; }
    uint32_t off;
    if (!b_mn) off = (kk / 64) * (N * 128) + tc::sw128_off(n, kk % 64);
    else off = (n / 64) * (K * 128) + tc::sw128_off(kk, n % 64);
    *reinterpret_cast<__nv_bfloat16*>(sbm + off) = val;
  }
  if (warp == 0) {
    tc::tmem_alloc(s_tmem, 256);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(mbar, 1);
    tc::fence_mbar_init();
  }
  tc::fence_proxy_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tm = *s_tmem;
  const uint32_t sa_u = tc::smem_u32(sa), sb_u = tc::smem_u32(sbm);
  if (tid == 0) {
    const uint32_t id = tc::idesc_f16(128, N, true, a_mn != 0, b_mn != 0);
    for (int ks = 0; ks < K / 16; ++ks) {
      uint64_t da, db;
      if (!a_mn) da = tc::desc_sw128(sa_u + (ks / 4) * (128 * 128) + (ks % 4) * 32, 16, 1024);
      else da = tc::desc_sw128(sa_u + ks * 2048, K * 128, 1024);
      if (!b_mn) db = tc::desc_sw128(sb_u + (ks / 4) * (N * 128) + (ks % 4) * 32, 16, 1024);
      else db = tc::desc_sw128(sb_u + ks * 2048, K * 128, 1024);
      tc::mma_f16(tm, da, db, id, ks > 0);
    }
    tc::mma_commit(mbar);
  }
  const bool ok = tc::mbar_wait(mbar, 0, kWaitLimit);
  tc::fence_after_sync();
  const int row = 32 * warp + lane;
  for (int c0 = 0; c0 < N; c0 += 32) {
    uint32_t r[32];
    tc::tmem_ld32(tm + ((uint32_t)(32 * warp) << 16) + c0, r);
    tc::tmem_wait_ld();
    for (int j = 0; j < 32; ++j) d[row * N + c0 + j] = ok ? __uint_as_float(r[j]) : NAN;
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tm, 256);
  }
}

}  // namespace
}  // namespace fo

using namespace fo;

namespace {
inline int64_t gdr_flags_bytes(int64_t heads) { return (heads * (int64_t)sizeof(int) + 255) & ~(int64_t)255; }

inline bool gdr_tc_eligible(const void* q, const void* k, const void* v, const void* o,
                            const float* hT, int64_t D, int dtype) {
  return (D == 16 || D == 32 || D == 64 || D == 128) && (dtype == FO_BF16 || dtype == FO_F16) &&
         aligned16(q) && aligned16(k) &&
         aligned16(v) && aligned16(o) && (!hT || aligned16(hT));
}
}  // namespace

extern "C" int fo_gdr_workspace_bytes(int64_t B, int64_t H, int64_t L, int64_t D, int dtype,
                                      int64_t* bytes) {
  clear_error();
  FO_CHECK_ARG(bytes && B >= 0 && H >= 0 && L >= 0, "fo_gdr_workspace_bytes: bad argument");
  // the tensor-core path: one int flag per head (fp16 range guard), then the
  // fp16 T tile of every (head, chunk) (8 KB each, 256-byte aligned)
  if ((D == 16 || D == 32 || D == 64 || D == 128) && (dtype == FO_BF16 || dtype == FO_F16)) {
    const int64_t nc = (L + kC - 1) / kC;
    *bytes = gdr_flags_bytes(B * H) + B * H * nc * 8192;
  } else {
    *bytes = 0;
  }
  return FO_OK;
}

extern "C" int fo_gdr_fwd(const void* q, const void* k, const void* v, const void* beta,
                          const void* g, const float* h0, void* o, float* hT, int64_t B, int64_t H,
                          int64_t L, int64_t D, int dtype, int gate_dtype, void* workspace,
                          int64_t ws_bytes, void* stream) {
  clear_error();
  FO_CHECK_ARG(B >= 0 && H >= 0 && L >= 0, "chunk_gated_delta_rule: negative size");
  if (D != 16 && D != 32 && D != 64 && D != 128) {
    set_error("D=%lld not in supported set {16,32,64,128}", (long long)D);
    return FO_EUNSUPPORTED;
  }
  if (B * H == 0) return FO_OK;
  FO_CHECK_ARG(!(h0 && hT && (const void*)h0 == (const void*)hT),
               "chunk_gated_delta_rule: initial and final state must not alias");
  cudaStream_t st = as_stream(stream);
  if (L == 0) {
    // no tokens: the final state is the initial one (the empty q, k, v, o may
    // have null data pointers)
    cudaError_t e = cudaSuccess;
    if (hT && h0)
      e = cudaMemcpyAsync(hT, h0, B * H * D * D * sizeof(float), cudaMemcpyDeviceToDevice, st);
    else if (hT)
      e = cudaMemsetAsync(hT, 0, B * H * D * D * sizeof(float), st);
    if (e != cudaSuccess) {
      set_error("chunk_gated_delta_rule: %s", cudaGetErrorString(e));
      return FO_ECUDA;
    }
    return FO_OK;
  }
  FO_CHECK_ARG(q && k && v && beta && g && o, "chunk_gated_delta_rule: null pointer");
  if (gdr_tc_eligible(q, k, v, o, hT, D, dtype)) {
    int64_t need = 0;
    fo_gdr_workspace_bytes(B, H, L, D, dtype, &need);
    if (!workspace || ws_bytes < need || !aligned16(workspace)) {
      set_error("chunk_gated_delta_rule: 16-byte-aligned workspace of %lld bytes required, got %lld",
                (long long)need, (long long)ws_bytes);
      return FO_EWORKSPACE;
    }
    int* flags = reinterpret_cast<int*>(workspace);
    __half* tbuf = reinterpret_cast<__half*>(reinterpret_cast<char*>(workspace) +
                                             gdr_flags_bytes(B * H));
    int rc = dtype == FO_BF16
                 ? tc_gate_dispatch<__nv_bfloat16>(gate_dtype, q, k, v, beta, g, h0, o, hT, flags,
                                                   tbuf, B * H, L, (int)D, st)
                 : tc_gate_dispatch<__half>(gate_dtype, q, k, v, beta, g, h0, o, hT, flags, tbuf,
                                            B * H, L, (int)D, st);
    if (rc) return rc;
    // heads whose fp16 operands left the fp16 range: exact fp32 per-step recomputation
    // (every other head's CTA returns at once)
    return gdr_stepwise(q, k, v, beta, g, h0, o, hT, B, H, L, D, dtype, gate_dtype, st, flags);
  }
  return gdr_stepwise(q, k, v, beta, g, h0, o, hT, B, H, L, D, dtype, gate_dtype, st);
}

extern "C" int fo_gdr_timeouts(unsigned int* count) {
  clear_error();
  FO_CHECK_ARG(count, "fo_gdr_timeouts: null pointer");
  if (cudaMemcpyFromSymbol(count, g_gdr_timeouts, sizeof(unsigned int)) != cudaSuccess) {
    set_error("fo_gdr_timeouts: cannot read the device counter");
    return FO_ECUDA;
  }
  return FO_OK;
}

extern "C" int fo_tc05_selftest(const void* a, const void* b, float* d, int64_t N, int64_t K,
                                int a_mn, int b_mn, void* stream) {
  clear_error();
  FO_CHECK_ARG(a && b && d, "fo_tc05_selftest: null pointer");
  FO_CHECK_ARG((N == 64 || N == 128) && (K == 64 || K == 128), "fo_tc05_selftest: N, K in {64,128}");
  const size_t smem = 128 * K * 2 + N * K * 2 + 64 + 1024;
  cudaFuncSetAttribute(tc_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  tc_selftest_kernel<<<1, 128, smem, as_stream(stream)>>>((const __nv_bfloat16*)a,
                                                          (const __nv_bfloat16*)b, d, (int)N,
                                                          (int)K, a_mn, b_mn);
  return check_launch("tc_selftest_kernel");
}
