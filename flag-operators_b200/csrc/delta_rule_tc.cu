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
#include <math.h>

#include "common.cuh"
#include "tc05.cuh"

namespace fo {
int gdr_stepwise(const void* q, const void* k, const void* v, const void* beta, const void* g,
                 const float* h0, void* o, float* hT, int64_t B, int64_t H, int64_t L, int64_t D,
                 int dtype, int gate_dtype, cudaStream_t st);

__device__ unsigned int g_gdr_timeouts;

namespace {

constexpr int kC = 64;
constexpr int kD = 128;
constexpr int kThr = 256;
constexpr uint32_t kWaitLimit = 1u << 22;

// shared-memory map (bytes from a 1024-aligned base)
constexpr uint32_t OFF_QK = 0;         // 2 x [128 x 128B]: rows 0-63 Q (later gQ), 64-127 K (later gK)
constexpr uint32_t OFF_V = 32768;      // 2 x [64 x 128B]
constexpr uint32_t OFF_KT = 49152;     // 2 x [64 x 128B]  Kt
constexpr uint32_t OFF_T = 65536;      // [64 x 128B]      T
constexpr uint32_t OFF_P = 73728;      // [64 x 128B]      P
constexpr uint32_t OFF_WT = 81920;     // [128 x 128B]     -W^T
constexpr uint32_t OFF_S = 98304;      // 2 x [128 x 128B] state (fp16 copy)
constexpr uint32_t OFF_UT = 131072;    // [128 x 128B]     U^T; then output staging [64 x 256B]
constexpr uint32_t OFF_RAW = 147456;   // [3][64 x 256B]   next chunk's q, k, v rows (bulk copy)
constexpr uint32_t OFF_A = 196608;     // fp32 [64][68]    A (rows 16-byte aligned)
constexpr uint32_t OFF_G = 214016;     // gate tables + barriers
constexpr int kAStride = 68;
constexpr uint32_t G_LC = 0, G_Z = 256, G_NEG = 512, G_BETA = 768, G_GAM = 1024, G_GAMP = 1280,
                   G_KTS = 1536, G_MISC = 1792;
constexpr uint32_t kSmemBytes = OFF_G + 2048 + 1024;  // + alignment slack

// TMEM columns (fp32 accumulators, 128 lanes)
constexpr uint32_t TM_S = 0, TM_U = 128, TM_O = 192, TM_QK = 256, TM_W = 320, TM_COLS = 512;

// element type of every tensor-core operand tile
using Op = __half;

// 8 input elements (16 bytes of T) -> 8 fp16 operand elements
template <typename T>
__device__ __forceinline__ uint4 to_op8(uint4 u) {
  if constexpr (std::is_same<T, __half>::value) {
    return u;
  } else {
    const T* e = reinterpret_cast<const T*>(&u);
    uint4 r;
    __half* h = reinterpret_cast<__half*>(&r);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = __float2half_rn(to_f<T>(e[i]));
    return r;
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  T x = from_f<T>(a), y = from_f<T>(b);
  return (uint32_t)(*reinterpret_cast<uint16_t*>(&x)) |
         ((uint32_t)(*reinterpret_cast<uint16_t*>(&y)) << 16);
}

// element-wise scale of a 16-byte chunk of 8 16-bit values
template <typename T>
__device__ __forceinline__ uint4 scale8(uint4 u, float s) {
  T* e = reinterpret_cast<T*>(&u);
  uint4 r;
  uint32_t* rr = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) rr[i] = pack2<Op>(to_f<T>(e[2 * i]) * s, to_f<T>(e[2 * i + 1]) * s);
  return r;
}

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
    const float r = expf(e);
    return par ? -r : r;
  }
};

__device__ __forceinline__ void cta_sync_tc() {
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
}

template <typename T, typename G>
__global__ void __launch_bounds__(kThr, 1)
gdr_tc_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
              const G* __restrict__ beta, const G* __restrict__ g, const float* __restrict__ h0,
              T* __restrict__ o, float* __restrict__ hT, int64_t L) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~(uintptr_t)1023);
  const uint32_t sb = tc::smem_u32(sm);
  float* sLc = reinterpret_cast<float*>(sm + OFF_G + G_LC);
  int* sZ = reinterpret_cast<int*>(sm + OFF_G + G_Z);
  int* sNeg = reinterpret_cast<int*>(sm + OFF_G + G_NEG);
  float* sBeta = reinterpret_cast<float*>(sm + OFF_G + G_BETA);
  float* sGam = reinterpret_cast<float*>(sm + OFF_G + G_GAM);
  float* sGamP = reinterpret_cast<float*>(sm + OFF_G + G_GAMP);
  float* sKts = reinterpret_cast<float*>(sm + OFF_G + G_KTS);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + OFF_G + G_MISC);
  uint64_t* rawbar = reinterpret_cast<uint64_t*>(sm + OFF_G + G_MISC + 8);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + OFF_G + G_MISC + 16);
  int* s_abort = reinterpret_cast<int*>(sm + OFF_G + G_MISC + 20);
  float* s_gc = reinterpret_cast<float*>(sm + OFF_G + G_MISC + 24);
  float* sA = reinterpret_cast<float*>(sm + OFF_A);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int quad = warp & 3, colh = warp >> 2;
  const int64_t head = blockIdx.x;
  const T* qh = q + head * L * kD;
  const T* kh = k + head * L * kD;
  const T* vh = v + head * L * kD;
  T* oh = o + head * L * kD;
  const G* bh = beta + head * L;
  const G* gh = g + head * L;
  constexpr bool BF = false;  // operands are fp16
  const GateTabs gt{sLc, sZ, sNeg};
  const int64_t nchunks = (L + kC - 1) / kC;

  if (warp == 0) {
    tc::tmem_alloc(s_tmem, TM_COLS);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(mbar, 1);
    tc::mbar_init(rawbar, 1);
    tc::fence_mbar_init();
    *s_abort = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tm = *s_tmem;
  const uint32_t tm_lane = tm + ((uint32_t)(32 * quad) << 16);
  uint32_t phase = 0, rphase = 0;
  bool state_nz = false;

  // q, k, v rows of chunk c -> RAW (bulk copies, completion on rawbar)
  auto issue_raw = [&](int64_t c) {
    const int64_t t0 = c * kC;
    const int nv = (int)((L - t0) < kC ? (L - t0) : kC);
    const uint32_t bytes = (uint32_t)nv * kD * sizeof(T);
    tc::mbar_arrive_expect_tx(rawbar, 3 * bytes);
    tc::bulk_g2s(sm + OFF_RAW, qh + t0 * kD, bytes, rawbar);
    tc::bulk_g2s(sm + OFF_RAW + 16384, kh + t0 * kD, bytes, rawbar);
    tc::bulk_g2s(sm + OFF_RAW + 32768, vh + t0 * kD, bytes, rawbar);
  };
  // thread 0 polls an mbarrier (bounded); the CTA barrier publishes the outcome
  auto bar_wait = [&](uint64_t* bar, uint32_t& ph) {
    if (tid == 0) {
      if (!tc::mbar_wait(bar, ph, kWaitLimit)) {
        atomicAdd(&g_gdr_timeouts, 1u);
        *s_abort = 1;
      }
    }
    ph ^= 1u;
    cta_sync_tc();
  };
  auto mma_wait = [&]() { bar_wait(mbar, phase); };

  if (tid == 0 && nchunks > 0) issue_raw(0);

  // ---- initial state
  if (h0) {
    const float* hh = h0 + head * kD * kD;
    const int i = 32 * quad + lane;  // state row (value channel)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int j0 = 64 * colh + 32 * half;
      uint32_t r[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(hh[i * kD + j0 + j]);
      tc::tmem_st32(tm_lane + TM_S + j0, r);
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint4 pk;
        pk.x = pack2<Op>(__uint_as_float(r[8 * c4 + 0]), __uint_as_float(r[8 * c4 + 1]));
        pk.y = pack2<Op>(__uint_as_float(r[8 * c4 + 2]), __uint_as_float(r[8 * c4 + 3]));
        pk.z = pack2<Op>(__uint_as_float(r[8 * c4 + 4]), __uint_as_float(r[8 * c4 + 5]));
        pk.w = pack2<Op>(__uint_as_float(r[8 * c4 + 6]), __uint_as_float(r[8 * c4 + 7]));
        *reinterpret_cast<uint4*>(sm + OFF_S + colh * 16384 + tc::sw128_chunk(i, 4 * half + c4)) =
            pk;
      }
    }
    tc::tmem_wait_st();
    state_nz = true;
  }

  for (int64_t c = 0; c < nchunks; ++c) {
    const int64_t tok0 = c * kC;
    const int nvalid = (int)((L - tok0) < kC ? (L - tok0) : kC);

    // ---- gates (small direct loads) while the bulk copy lands
    if (tid < 64) {
      const bool ok = tid < nvalid;
      const float bt = ok ? to_f<G>(bh[tok0 + tid]) : 0.f;
      const float gg = ok ? to_f<G>(gh[tok0 + tid]) : 1.f;
      sBeta[tid] = bt;
      // prefix sums over the chunk: log|g|, last zero-gate index, negative count
      float lg = (gg != 0.f) ? logf(fabsf(gg)) : 0.f;
      int zi = (gg == 0.f) ? tid : -1;
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
      sLc[tid] = lg;
      sZ[tid] = zi;
      sNeg[tid] = ng;
    }
    bar_wait(rawbar, rphase);  // includes a CTA barrier
    if (*s_abort) break;
    if (tid >= 32 && tid < 64) {
      sLc[tid] += sLc[31];
      sZ[tid] = max(sZ[tid], sZ[31]);
      sNeg[tid] += sNeg[31];
    }
    // RAW (T, row-major) -> fp16 swizzled operand tiles; rows past the end are zero
    for (int idx = tid; idx < 3 * 1024; idx += kThr) {
      const int m = idx >> 10, rem = idx & 1023, t = rem >> 4, ch = rem & 15;
      const int half = ch >> 3, cc = ch & 7;
      uint4 val = make_uint4(0, 0, 0, 0);
      if (t < nvalid)
        val = to_op8<T>(*reinterpret_cast<const uint4*>(sm + OFF_RAW + m * 16384 + t * 256 + ch * 16));
      uint32_t off;
      if (m == 0) off = OFF_QK + half * 16384 + tc::sw128_chunk(t, cc);
      else if (m == 1) off = OFF_QK + half * 16384 + tc::sw128_chunk(64 + t, cc);
      else off = OFF_V + half * 8192 + tc::sw128_chunk(t, cc);
      *reinterpret_cast<uint4*>(sm + off) = val;
    }
    __syncthreads();
    if (tid == 0 && c + 1 < nchunks) {
      tc::fence_proxy_async();  // RAW was read through the generic proxy
      issue_raw(c + 1);
    }
    if (tid < 64) {
      sGam[tid] = gt.ratio(tid, -1);
      sGamP[tid] = tid > 0 ? gt.ratio(tid - 1, -1) : 1.f;
      sKts[tid] = gt.ratio(kC - 1, tid) * sBeta[tid];
      if (tid == 0) *s_gc = gt.ratio(kC - 1, -1);
    }
    tc::fence_proxy_async();
    cta_sync_tc();

    // ---- (a) [Q;K] K^T -> TM_QK
    if (tid == 0) {
      constexpr uint32_t id_a = tc::idesc_f16(128, 64, BF, false, false);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t h = ks >> 2, kk = ks & 3;
        const uint64_t da = tc::desc_sw128(sb + OFF_QK + h * 16384 + kk * 32, 16, 1024);
        const uint64_t db = tc::desc_sw128(sb + OFF_QK + h * 16384 + 8192 + kk * 32, 16, 1024);
        tc::mma_f16(tm + TM_QK, da, db, id_a, ks > 0);
      }
      tc::mma_commit(mbar);
    }
    mma_wait();
    if (*s_abort) break;

    // ---- P (rows 0-63) and A (rows 64-127) from the QK / KK block
    {
      uint32_t r[32];
      tc::tmem_ld32(tm_lane + TM_QK + 32 * colh, r);
      tc::tmem_wait_ld();
      const int row = 32 * quad + lane;
      if (row < 64) {
        const int t = row;
        float pv[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int s = 32 * colh + j;
          pv[j] = (s <= t) ? gt.ratio(t, s) * sBeta[s] * __uint_as_float(r[j]) : 0.f;
        }
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint4 pk;
          pk.x = pack2<Op>(pv[8 * c4 + 0], pv[8 * c4 + 1]);
          pk.y = pack2<Op>(pv[8 * c4 + 2], pv[8 * c4 + 3]);
          pk.z = pack2<Op>(pv[8 * c4 + 4], pv[8 * c4 + 5]);
          pk.w = pack2<Op>(pv[8 * c4 + 6], pv[8 * c4 + 7]);
          *reinterpret_cast<uint4*>(sm + OFF_P + tc::sw128_chunk(t, 4 * colh + c4)) = pk;
        }
      } else {
        const int t = row - 64;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int s = 32 * colh + j;
          sA[t * kAStride + s] =
              (s < t) ? gt.ratio(t - 1, s) * sBeta[s] * __uint_as_float(r[j]) : 0.f;
        }
      }
    }
    cta_sync_tc();

    if (tid < 64) {
      // ---- T = (I + A)^-1 by forward substitution, one column per thread:
      //      T[i][j] = [i == j] - sum_{m < i} A[i][m] T[m][j]
      // The column lives in registers; row i of A is a broadcast read.
      const int j = tid;
      float col[kC];
#pragma unroll
      for (int i = 0; i < kC; ++i) {
        float acc0 = (i == j) ? 1.f : 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
#pragma unroll
        for (int m = 0; m < i; m += 4) {
          const float4 a4 = *reinterpret_cast<const float4*>(sA + i * kAStride + m);
          acc0 = fmaf(-a4.x, col[m], acc0);
          if (m + 1 < i) acc1 = fmaf(-a4.y, col[m + 1], acc1);
          if (m + 2 < i) acc2 = fmaf(-a4.z, col[m + 2], acc2);
          if (m + 3 < i) acc3 = fmaf(-a4.w, col[m + 3], acc3);
        }
        col[i] = (acc0 + acc1) + (acc2 + acc3);
      }
      // column j of T -> fp16 tile [t][s] (K-major B operand of (b), (c))
      __half* tt = reinterpret_cast<__half*>(sm + OFF_T);
#pragma unroll
      for (int i = 0; i < kC; ++i)
        *reinterpret_cast<__half*>(sm + OFF_T + tc::sw128_off(i, j)) = __float2half_rn(col[i]);
      (void)tt;
    } else {
      // ---- scaled copies (other 6 warps): gQ (in place), Kt (new), gK (in place)
      for (int idx = tid - 64; idx < 2048; idx += kThr - 64) {
        const int m = idx >> 10, rem = idx & 1023, t = rem >> 4, ch = rem & 15;
        const int half = ch >> 3, cc = ch & 7;
        if (m == 0) {
          uint4* pp = reinterpret_cast<uint4*>(sm + OFF_QK + half * 16384 + tc::sw128_chunk(t, cc));
          *pp = scale8<Op>(*pp, sGam[t]);
        } else {
          uint4* pp =
              reinterpret_cast<uint4*>(sm + OFF_QK + half * 16384 + tc::sw128_chunk(64 + t, cc));
          const uint4 raw = *pp;
          *reinterpret_cast<uint4*>(sm + OFF_KT + half * 8192 + tc::sw128_chunk(t, cc)) =
              scale8<Op>(raw, sKts[t]);
          *pp = scale8<Op>(raw, sGamP[t]);
        }
      }
    }
    tc::fence_proxy_async();
    cta_sync_tc();
    // ---- (b) W^T = (gK)^T T^T,  (c) U^T = V^T T^T
    if (tid == 0) {
      constexpr uint32_t id_mn = tc::idesc_f16(128, 64, BF, true, false);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint64_t dt = tc::desc_sw128(sb + OFF_T + ks * 32, 16, 1024);
        const uint64_t dk = tc::desc_sw128(sb + OFF_QK + 8192 + ks * 2048, 16384, 1024);
        const uint64_t dv = tc::desc_sw128(sb + OFF_V + ks * 2048, 8192, 1024);
        tc::mma_f16(tm + TM_W, dk, dt, id_mn, ks > 0);
        tc::mma_f16(tm + TM_U, dv, dt, id_mn, ks > 0);
      }
      tc::mma_commit(mbar);
    }
    mma_wait();
    if (*s_abort) break;

    // ---- -W^T -> bf16 tile [j][t] (MN-major B operand of (d))
    {
      uint32_t r[32];
      tc::tmem_ld32(tm_lane + TM_W + 32 * colh, r);
      tc::tmem_wait_ld();
      const int j = 32 * quad + lane;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint4 pk;
        pk.x = pack2<Op>(-__uint_as_float(r[8 * c4 + 0]), -__uint_as_float(r[8 * c4 + 1]));
        pk.y = pack2<Op>(-__uint_as_float(r[8 * c4 + 2]), -__uint_as_float(r[8 * c4 + 3]));
        pk.z = pack2<Op>(-__uint_as_float(r[8 * c4 + 4]), -__uint_as_float(r[8 * c4 + 5]));
        pk.w = pack2<Op>(-__uint_as_float(r[8 * c4 + 6]), -__uint_as_float(r[8 * c4 + 7]));
        *reinterpret_cast<uint4*>(sm + OFF_WT + tc::sw128_chunk(j, 4 * colh + c4)) = pk;
      }
    }
    tc::fence_proxy_async();
    cta_sync_tc();

    // ---- (d) U^T += S (-W)^T,  (e) O^T = S (gQ)^T
    if (state_nz) {
      if (tid == 0) {
        constexpr uint32_t id_d = tc::idesc_f16(128, 64, BF, false, true);
        constexpr uint32_t id_e = tc::idesc_f16(128, 64, BF, false, false);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t h = ks >> 2, kk = ks & 3;
          const uint64_t ds = tc::desc_sw128(sb + OFF_S + h * 16384 + kk * 32, 16, 1024);
          const uint64_t dw = tc::desc_sw128(sb + OFF_WT + ks * 2048, 8192, 1024);
          const uint64_t dq = tc::desc_sw128(sb + OFF_QK + h * 16384 + kk * 32, 16, 1024);
          tc::mma_f16(tm + TM_U, ds, dw, id_d, 1);
          tc::mma_f16(tm + TM_O, ds, dq, id_e, ks > 0);
        }
        tc::mma_commit(mbar);
      }
      mma_wait();
      if (*s_abort) break;
    }

    // ---- U^T -> bf16 tile [i][s]; decay the fp32 state by gamma_{C-1}
    {
      uint32_t r[32];
      tc::tmem_ld32(tm_lane + TM_U + 32 * colh, r);
      tc::tmem_wait_ld();
      const int i = 32 * quad + lane;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint4 pk;
        pk.x = pack2<Op>(__uint_as_float(r[8 * c4 + 0]), __uint_as_float(r[8 * c4 + 1]));
        pk.y = pack2<Op>(__uint_as_float(r[8 * c4 + 2]), __uint_as_float(r[8 * c4 + 3]));
        pk.z = pack2<Op>(__uint_as_float(r[8 * c4 + 4]), __uint_as_float(r[8 * c4 + 5]));
        pk.w = pack2<Op>(__uint_as_float(r[8 * c4 + 6]), __uint_as_float(r[8 * c4 + 7]));
        *reinterpret_cast<uint4*>(sm + OFF_UT + tc::sw128_chunk(i, 4 * colh + c4)) = pk;
      }
      if (state_nz) {
        const float gc = *s_gc;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const uint32_t col = TM_S + 64 * colh + 32 * hf;
          tc::tmem_ld32(tm_lane + col, r);
          tc::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * gc);
          tc::tmem_st32(tm_lane + col, r);
        }
        tc::tmem_wait_st();
      }
    }
    tc::fence_proxy_async();
    cta_sync_tc();

    // ---- (f) O^T += U^T P^T,  (g) S (+)= U^T Kt
    if (tid == 0) {
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
      tc::mma_commit(mbar);
    }
    mma_wait();
    if (*s_abort) break;
    state_nz = true;

    // ---- outputs: O^T -> o rows (staged row-major), state -> bf16 operand tile
    {
      uint32_t r[32];
      tc::tmem_ld32(tm_lane + TM_O + 32 * colh, r);
      tc::tmem_wait_ld();
      const int i = 32 * quad + lane;
      T* so = reinterpret_cast<T*>(sm + OFF_UT);
#pragma unroll
      for (int j = 0; j < 32; ++j) so[(32 * colh + j) * kD + i] = from_f<T>(__uint_as_float(r[j]));
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        tc::tmem_ld32(tm_lane + TM_S + 64 * colh + 32 * hf, r);
        tc::tmem_wait_ld();
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint4 pk;
          pk.x = pack2<Op>(__uint_as_float(r[8 * c4 + 0]), __uint_as_float(r[8 * c4 + 1]));
          pk.y = pack2<Op>(__uint_as_float(r[8 * c4 + 2]), __uint_as_float(r[8 * c4 + 3]));
          pk.z = pack2<Op>(__uint_as_float(r[8 * c4 + 4]), __uint_as_float(r[8 * c4 + 5]));
          pk.w = pack2<Op>(__uint_as_float(r[8 * c4 + 6]), __uint_as_float(r[8 * c4 + 7]));
          *reinterpret_cast<uint4*>(sm + OFF_S + colh * 16384 +
                                    tc::sw128_chunk(i, 4 * hf + c4)) = pk;
        }
      }
    }
    tc::fence_proxy_async();
    cta_sync_tc();
    for (int e = tid; e < nvalid * 16; e += kThr) {
      const int t = e >> 4, ch = e & 15;
      st_global_v4(oh + (tok0 + t) * kD + ch * 8,
                   *reinterpret_cast<const uint4*>(sm + OFF_UT + t * 256 + ch * 16));
    }
    // (next chunk's loads overwrite QK/V/KT only after the barrier that follows them)
  }

  // an abort can leave one bulk copy in flight: let it land before the CTA exits
  if (*s_abort && tid == 0) tc::mbar_wait(rawbar, rphase, kWaitLimit);

  // ---- final state
  if (hT && !*s_abort) {
    float* hh = hT + head * kD * kD;
    const int i = 32 * quad + lane;
    for (int hf = 0; hf < 2; ++hf) {
      uint32_t r[32];
      const int j0 = 64 * colh + 32 * hf;
      if (state_nz) {
        tc::tmem_ld32(tm_lane + TM_S + j0, r);
        tc::tmem_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;
      }
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4)
        *reinterpret_cast<uint4*>(hh + i * kD + j0 + 4 * j4) =
            make_uint4(r[4 * j4], r[4 * j4 + 1], r[4 * j4 + 2], r[4 * j4 + 3]);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tm, TM_COLS);
  }
}

template <typename T, typename G>
int launch_tc(const void* q, const void* k, const void* v, const void* beta, const void* g,
              const float* h0, void* o, float* hT, int64_t BH, int64_t L, cudaStream_t st) {
  auto kern = gdr_tc_kernel<T, G>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
      cudaSuccess) {
    set_error("gdr_tc_kernel: cannot reserve %u bytes of shared memory", kSmemBytes);
    return FO_ECUDA;
  }
  kern<<<(unsigned)BH, kThr, kSmemBytes, st>>>((const T*)q, (const T*)k, (const T*)v,
                                               (const G*)beta, (const G*)g, h0, (T*)o, hT, L);
  return check_launch("gdr_tc_kernel");
}

template <typename T>
int tc_gate_dispatch(int gate_dtype, const void* q, const void* k, const void* v, const void* beta,
                     const void* g, const float* h0, void* o, float* hT, int64_t BH, int64_t L,
                     cudaStream_t st) {
  switch (gate_dtype) {
    case FO_F32: return launch_tc<T, float>(q, k, v, beta, g, h0, o, hT, BH, L, st);
    case FO_F16: return launch_tc<T, __half>(q, k, v, beta, g, h0, o, hT, BH, L, st);
    case FO_BF16: return launch_tc<T, __nv_bfloat16>(q, k, v, beta, g, h0, o, hT, BH, L, st);
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

extern "C" int fo_gdr_fwd(const void* q, const void* k, const void* v, const void* beta,
                          const void* g, const float* h0, void* o, float* hT, int64_t B, int64_t H,
                          int64_t L, int64_t D, int dtype, int gate_dtype, void* stream) {
  clear_error();
  FO_CHECK_ARG(B >= 0 && H >= 0 && L >= 0, "chunk_gated_delta_rule: negative size");
  if (D != 16 && D != 32 && D != 64 && D != 128) {
    set_error("D=%lld not in supported set {16,32,64,128}", (long long)D);
    return FO_EUNSUPPORTED;
  }
  if (B * H == 0) return FO_OK;
  FO_CHECK_ARG(q && k && v && beta && g && o, "chunk_gated_delta_rule: null pointer");
  cudaStream_t st = as_stream(stream);
  if (L == 0) {
    if (hT && h0)
      cudaMemcpyAsync(hT, h0, B * H * D * D * sizeof(float), cudaMemcpyDeviceToDevice, st);
    else if (hT)
      cudaMemsetAsync(hT, 0, B * H * D * D * sizeof(float), st);
    return FO_OK;
  }
  const bool tc_ok = D == 128 && (dtype == FO_BF16 || dtype == FO_F16) && aligned16(q) &&
                     aligned16(k) && aligned16(v) && aligned16(o) && (!hT || aligned16(hT));
  if (tc_ok) {
    if (dtype == FO_BF16)
      return tc_gate_dispatch<__nv_bfloat16>(gate_dtype, q, k, v, beta, g, h0, o, hT, B * H, L, st);
    return tc_gate_dispatch<__half>(gate_dtype, q, k, v, beta, g, h0, o, hT, B * H, L, st);
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
