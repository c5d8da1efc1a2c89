// Gated-delta-rule suffix replay from a shared, request-sized state (beam decode).
//
// Semantics: src/kadllm/ops.py:139-163 (torch path of gated_delta) and the
// Triton kernels src/kadllm/kernels/gated_delta.py:14-142 it accelerates.  Every
// beam of request b starts from the same immutable state S0 = state[b, hv]
// (K x V) and replays T <= 8 suffix tokens:
//     S <- S * exp(g_t);  d_t = beta_t (v_t - S^T k_t);  S <- S + k_t d_t^T;  o_t = S^T q_t
// with q, k L2-normalised (eps 1e-6 inside the sqrt) and q scaled.
//
// B200 formulation (no per-beam state copy): unrolling the recurrence gives
//     S_t'^T k_t = A_t (S0^T k_t) + sum_{s<t} D(s,t) d_s (k_s . k_t)
//     o_t        = A_t (S0^T q_t) + sum_{s<=t} D(s,t) d_s (k_s . q_t)
//     A_t = prod_{r<=t} a_r,  D(s,t) = prod_{s<r<=t} a_r,  a_r = exp(g_r),
// so the only K x V work is multiplying the beams' q_t / k_t rows by S0, which
// runs on the tensor cores with S0 staged once in shared memory.
//
// Thread mapping: a warp owns 8 beams, thread quad g one beam.  For step t the
// warp's 16 rows [q_t of the 8 beams ; k_t of the 8 beams] go to tensor memory
// (lanes 32w + g and 32w + 8 + g, 16x256b stores) and one thread runs the
// CTA's tcgen05 MMAs (M = 128: the warps' row blocks, N = V) against S0 staged
// once as an MN-major shared-memory operand; the 16x256b loads of the
// accumulator give thread (g, tq) S0^T q_t and S0^T k_t of beam g for the
// columns {8j + 2tq, 8j + 2tq + 1}: the recurrence, the output cast and (fused
// mixer) the gated RMSNorm are thread-local plus two quad shuffles.  The warps
// of a CTA advance in lock step, one (octet, step) per round.  q/k are split
// into bf16 hi + lo parts (A = A_hi + A_lo, and S0 too when it is not bf16:
// A_hi S_hi + A_lo S_hi + A_hi S_lo), keeping ~16 mantissa bits in the
// products.  The contraction order is a bit permutation of the key index: the
// thread's pairs at keys 16kk + 8hp + 2tq + {0, 1} sit in TMEM column
// 8kk + 2tq + hp, i.e. MMA k index 16kk + 4tq + 2hp + {0, 1}, and S0's rows are
// staged in that order.  Earlier steps' k_s and d_s (T > 1) live in a small
// per-warp shared-memory slab.  The MMA completion wait is bounded and reports
// through the status word.
//
// Fused mixer (kadllm_gdn_mixer_replay): q/k/v are produced on the fly by the
// causal conv1d replay + SiLU from the packed projection row and the request's
// conv state (src/kadllm/kernels/causal_conv1d.py:41-48), the gates from the
// b / a columns (src/kadllm/adapters/qwen3_5.py:161-169), and the output goes
// through Qwen3_5RMSNormGated with z (transformers modeling_qwen3_5.py:175-190).
#include "common.cuh"
#include "gdn_mixer.cuh"
#include "tcgen05.cuh"

namespace kb {
namespace {

constexpr int kTMax = 8;
constexpr int kBeamsPerWarp = 8;

struct GdnArgs {
  // standalone operator inputs
  const void* q;
  const void* k;
  const void* v;
  int x_dtype;
  const void* g;
  int g_dtype;
  const void* beta;
  int beta_dtype;
  // fused mixer inputs
  const __nv_bfloat16* proj;
  int64_t ld_proj;
  const __nv_bfloat16* conv_state;
  int64_t conv_hist;
  const __nv_bfloat16* conv_weight;
  const float* a_log;
  const float* dt_bias;
  const float* norm_weight;
  float norm_eps;
  // common
  const void* state;
  int state_dtype;
  int state_split;  // 1: S0 needs a lo part (not bf16)
  void* out;
  int out_dtype;
  uint32_t* status;
  int B, W, T, H, HV;
  float scale;
  int octets_per_warp;  // beam octets each warp processes (amortises the S0 staging)
};

template <int DK, int DV>
struct Layout {
  static constexpr int NCH = 2 * DK + DV;   // conv channels of one (q head, k head, v head)
  static constexpr int KGRP = 16 * DV;      // bytes per group of 8 state rows in the operand image
  static constexpr int IMG = DK * DV * 2;   // one bf16 operand image of S0
  static constexpr int TCOLS = DV + DK;     // TMEM columns: accumulator, A hi, A lo
  static_assert(TCOLS == 64 || TCOLS == 128 || TCOLS == 256, "TMEM allocation is a power of two");
  // S0 image(s), then the mbarrier and the TMEM address slot (16 bytes)
  __host__ __device__ static size_t state_bytes(bool split) { return size_t(IMG) * (split ? 2 : 1) + 16; }
  __host__ __device__ static size_t conv_bytes(bool fused) { return fused ? size_t(NCH) * 8 * 4 : 0; }
  // per warp: k_s (fp32) and d_s (fp32) of the steps before the last, plus the
  // current step's bf16 outputs (read back by the gated RMSNorm)
  __host__ __device__ static size_t warp_bytes(int T) {
    return size_t(T > 1 ? T - 1 : 0) * kBeamsPerWarp * (DK + DV) * 4 + size_t(kBeamsPerWarp) * DV * 2;
  }
};

// conv channel table, component-major [8][NCH]: c0, c1, c2 (prefix-tap partial sums
// for t = 0, 1, 2), then w0..w3, so that for suffix step t
//   conv_t = c_t + sum_{s = max(0, t-3)}^{t} w_{3-(t-s)} x_s      (c_t = 0 for t >= 3).
// Evaluates two adjacent channels (c, c+1) from bf16 pairs of the projection rows.
template <int NCH>
__device__ __forceinline__ float2 conv_pair(const float* tab, int c, int t, const __nv_bfloat16* col0,
                                            int64_t row_stride) {
  float2 acc = t < 3 ? *reinterpret_cast<const float2*>(tab + t * NCH + c) : make_float2(0.f, 0.f);
  const int s0 = t > 3 ? t - 3 : 0;
  for (int s = s0; s <= t; ++s) {
    const float2 w = *reinterpret_cast<const float2*>(tab + (3 + 3 - (t - s)) * NCH + c);
    const __nv_bfloat162 x = *reinterpret_cast<const __nv_bfloat162*>(col0 + s * row_stride);
    acc.x += w.x * __low2float(x);
    acc.y += w.y * __high2float(x);
  }
  return acc;
}

// TMAX: compile-time bound on T (1, 2, 4 or 8) so the per-step loops carry no dead code.
// MMA k index (B row) of key r = 16kk + 8hp + 2tq + d: 16kk + 4tq + 2hp + d.
__device__ __forceinline__ int replay_kappa(int r) {
  return (r & ~15) | (((r >> 3) & 1) << 1) | (((r >> 1) & 3) << 2) | (r & 1);
}

template <int DK, int DV, bool FUSED, int TMAX>
__global__ void __launch_bounds__(128) gdn_replay_kernel(const GdnArgs a) {
  using Lt = Layout<DK, DV>;
  constexpr int KK = DK / 16;  // k16 steps (= 8-column TMEM blocks of one A part)
  constexpr int NT = DV / 8;   // n8 tiles
  constexpr long long kWait = 1ll << 31;
  constexpr uint32_t kIdesc = tc::idesc_bf16(128, DV, 0, 1);  // A (TMEM) x MN-major S0
  extern __shared__ __align__(16) unsigned char smem[];
  const int nwarps = blockDim.x >> 5;
  const int T = a.T;
  unsigned char* p = smem;
  unsigned char* sS = p;  // S0 hi image [, lo image]
  uint64_t* mbar = reinterpret_cast<uint64_t*>(p + Lt::IMG * (a.state_split ? 2 : 1));
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mbar + 1);
  p += Lt::state_bytes(a.state_split);
  float* sConv = reinterpret_cast<float*>(p);  // [NCH][8]
  p += Lt::conv_bytes(FUSED);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* sK = reinterpret_cast<float*>(p + warp * Lt::warp_bytes(T));  // [T-1][8][DK]
  float* sD = sK + (T > 1 ? T - 1 : 0) * kBeamsPerWarp * DK;           // [T-1][8][DV]
  __nv_bfloat16* sO = reinterpret_cast<__nv_bfloat16*>(sD + (T > 1 ? T - 1 : 0) * kBeamsPerWarp * DV);  // [8][DV]

  const int HV = a.HV;
  const int b = blockIdx.x / HV, hv = blockIdx.x % HV;
  const int h = hv / (HV / a.H);
  const int key_dim = a.H * DK;
  const int conv_dim = 2 * key_dim + HV * DV;
  const int g = lane >> 2, tq = lane & 3;

  // ---- TMEM, S0 (bf16 hi [+ lo] MN-major operand images) and the conv table ----------
  if (warp == 0) tc::tmem_alloc(tslot, Lt::TCOLS);
  if (tid == 0) {
    tc::mbar_init(mbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  {
    const int64_t base = (int64_t(b) * HV + hv) * DK * DV;
    for (int i = tid * 8; i < DK * DV; i += blockDim.x * 8) {  // 8 consecutive V columns of one key row
      float f[8];
      load4(a.state, base + i, a.state_dtype, f);
      load4(a.state, base + i + 4, a.state_dtype, f + 4);
      const int kr = i / DV, kap = replay_kappa(kr);
      const size_t off = size_t(kap >> 3) * Lt::KGRP + ((i % DV) >> 3) * 128 + (kap & 7) * 16;
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        hi[e] = pack_bf16(f[2 * e], f[2 * e + 1]);
        const float2 hf = bf2f(hi[e]);
        lo[e] = pack_bf16(f[2 * e] - hf.x, f[2 * e + 1] - hf.y);
      }
      *reinterpret_cast<uint4*>(sS + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      if (a.state_split) *reinterpret_cast<uint4*>(sS + Lt::IMG + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    if constexpr (FUSED) {
      for (int c = tid; c < Lt::NCH; c += blockDim.x) {
        int ch;
        if (c < DK) ch = h * DK + c;
        else if (c < 2 * DK) ch = key_dim + h * DK + (c - DK);
        else ch = 2 * key_dim + hv * DV + (c - 2 * DK);
        const __nv_bfloat16* w = a.conv_weight + int64_t(ch) * 4;
        const __nv_bfloat16* s = a.conv_state + (int64_t(b) * conv_dim + ch) * a.conv_hist + a.conv_hist - 3;
        const float w0 = __bfloat162float(w[0]), w1 = __bfloat162float(w[1]);
        const float w2 = __bfloat162float(w[2]), w3 = __bfloat162float(w[3]);
        const float s0 = __bfloat162float(s[0]), s1 = __bfloat162float(s[1]), s2 = __bfloat162float(s[2]);
        sConv[0 * Lt::NCH + c] = w0 * s0 + w1 * s1 + w2 * s2;
        sConv[1 * Lt::NCH + c] = w0 * s1 + w1 * s2;
        sConv[2 * Lt::NCH + c] = w0 * s2;
        sConv[3 * Lt::NCH + c] = w0;  // tap applied to x_{t-3}
        sConv[4 * Lt::NCH + c] = w1;
        sConv[5 * Lt::NCH + c] = w2;
        sConv[6 * Lt::NCH + c] = w3;  // tap applied to x_t
        sConv[7 * Lt::NCH + c] = 0.f;
      }
    }
  }
  tc::fence_async_smem();  // the operand images, visible to the tensor cores
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t t_acc = tc::taddr(tmem, 32 * warp, 0);  // this warp's 16 lanes: q rows g, k rows 8 + g
  const uint32_t t_hi = tc::taddr(tmem, 32 * warp, DV), t_lo = tc::taddr(tmem, 32 * warp, DV + DK / 2);
  const uint32_t s_img = smem_u32(sS);
  uint32_t round = 0;
  bool ok = true;

  for (int oct = 0; oct < a.octets_per_warp; ++oct) {
  const int beam = ((blockIdx.y * nwarps + warp) * a.octets_per_warp + oct) * kBeamsPerWarp + g;
  const bool valid = beam < a.W;
  const int64_t brow = int64_t(b) * a.W + (valid ? beam : 0);
  float At = 1.f;
  float Dst[TMAX];
  float kqd[TMAX], kkd[TMAX];  // k_s . q_t and k_s . k_t for the earlier steps s < t
#pragma unroll
  for (int s = 0; s < TMAX; ++s) Dst[s] = kqd[s] = kkd[s] = 0.f;

#pragma unroll
  for (int t = 0; t < TMAX; ++t) {
    if (t >= T) break;
    const int64_t row = brow * T + t;
    // ---- q_t, k_t, v_t of beam g at this thread's columns ---------------------------
    float qv[KK][4], kv[KK][4];
    float gt = 0.f, bt = 0.f;
#pragma unroll
    for (int kk = 0; kk < KK; ++kk)
#pragma unroll
      for (int hp = 0; hp < 2; ++hp) {  // column pairs (2tq, 2tq+1) and (2tq+8, 2tq+9)
        const int col = kk * 16 + tq * 2 + hp * 8;
        float2 qx = make_float2(0.f, 0.f), kx = make_float2(0.f, 0.f);
        if (valid) {
          if constexpr (FUSED) {
            const __nv_bfloat16* base = a.proj + (brow * T) * a.ld_proj;
            qx = conv_pair<Lt::NCH>(sConv, col, t, base + h * DK + col, a.ld_proj);
            kx = conv_pair<Lt::NCH>(sConv, DK + col, t, base + key_dim + h * DK + col, a.ld_proj);
            qx = make_float2(bf16r(silu_fast(qx.x)), bf16r(silu_fast(qx.y)));
            kx = make_float2(bf16r(silu_fast(kx.x)), bf16r(silu_fast(kx.y)));
          } else {
            const int64_t o = (row * a.H + h) * DK + col;
            qx = load2_as_float(a.q, o, a.x_dtype);
            kx = load2_as_float(a.k, o, a.x_dtype);
          }
        }
        qv[kk][2 * hp] = qx.x;
        qv[kk][2 * hp + 1] = qx.y;
        kv[kk][2 * hp] = kx.x;
        kv[kk][2 * hp + 1] = kx.y;
      }
    if (valid) {
      if constexpr (FUSED) {
        const __nv_bfloat16* pr = a.proj + row * a.ld_proj + conv_dim + int64_t(HV) * DV;
        bt = bf16r(sigmoid_f(__bfloat162float(pr[hv])));
        gt = -expf(a.a_log[hv]) * softplus_f(__bfloat162float(pr[HV + hv]) + a.dt_bias[hv]);
      } else {
        gt = load_as_float(a.g, row * HV + hv, a.g_dtype);
        bt = load_as_float(a.beta, row * HV + hv, a.beta_dtype);
      }
    }
    // ---- L2 norms (quad reduction: the 4 threads of a beam hold all K columns) -------
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int kk = 0; kk < KK; ++kk)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        sq += qv[kk][e] * qv[kk][e];
        sk += kv[kk][e] * kv[kk][e];
      }
    sq += __shfl_xor_sync(0xffffffffu, sq, 1);
    sq += __shfl_xor_sync(0xffffffffu, sq, 2);
    sk += __shfl_xor_sync(0xffffffffu, sk, 1);
    sk += __shfl_xor_sync(0xffffffffu, sk, 2);
    const float iq = 1.0f / sqrtf(sq + 1e-6f), ik = 1.0f / sqrtf(sk + 1e-6f);
#pragma unroll
    for (int kk = 0; kk < KK; ++kk)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        qv[kk][e] = qv[kk][e] * iq * a.scale;
        kv[kk][e] = kv[kk][e] * ik;
      }
    // ---- dot products with this beam's earlier keys ------------------------------------
    float kq_self;
    {
      float dqq = 0.f;
#pragma unroll
      for (int kk = 0; kk < KK; ++kk)
#pragma unroll
        for (int e = 0; e < 4; ++e) dqq += kv[kk][e] * qv[kk][e];
      dqq += __shfl_xor_sync(0xffffffffu, dqq, 1);
      dqq += __shfl_xor_sync(0xffffffffu, dqq, 2);
#pragma unroll
      for (int s = 0; s < t; ++s) {
        {
          const float* ks = sK + (s * kBeamsPerWarp + g) * DK;
          float dks = 0.f, dqs = 0.f;
#pragma unroll
          for (int kk = 0; kk < KK; ++kk)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float kse = ks[kk * 16 + tq * 2 + (e & 1) + (e >> 1) * 8];
              dks += kse * kv[kk][e];
              dqs += kse * qv[kk][e];
            }
          dks += __shfl_xor_sync(0xffffffffu, dks, 1);
          dks += __shfl_xor_sync(0xffffffffu, dks, 2);
          dqs += __shfl_xor_sync(0xffffffffu, dqs, 1);
          dqs += __shfl_xor_sync(0xffffffffu, dqs, 2);
          kkd[s] = dks;
          kqd[s] = dqs;
        }
      }
      kq_self = dqq;
    }
    // ---- P = [q_t ; k_t] x S0 on the tensor cores, then the factored recurrence ----
    // The V columns are processed in two halves to bound the accumulator registers.
    const float at = expf(gt);
    At *= at;
#pragma unroll
    for (int s = 0; s < t; ++s) Dst[s] *= at;
    constexpr int NH = NT / 2;
    float ss = 0.f;  // sum of squares of the bf16 outputs (fused gated norm)
    float* dcur = sD + (t * kBeamsPerWarp + g) * DV;
    // [q_t ; k_t] (lanes g / g + 8) into TMEM as bf16 hi and lo parts; thread 0 runs the MMAs
    {
      uint32_t ahi[4 * KK], alo[4 * KK];
#pragma unroll
      for (int kk = 0; kk < KK; ++kk)
#pragma unroll
        for (int hp = 0; hp < 2; ++hp) {  // TMEM column 8kk + 2tq + hp: keys 16kk + 8hp + 2tq + {0, 1}
          const float q0 = qv[kk][2 * hp], q1 = qv[kk][2 * hp + 1];
          const float k0 = kv[kk][2 * hp], k1 = kv[kk][2 * hp + 1];
          const float hq0 = bf16r(q0), hq1 = bf16r(q1), hk0 = bf16r(k0), hk1 = bf16r(k1);
          ahi[4 * kk + hp] = pack_bf16(hq0, hq1);
          ahi[4 * kk + 2 + hp] = pack_bf16(hk0, hk1);
          alo[4 * kk + hp] = pack_bf16(q0 - hq0, q1 - hq1);
          alo[4 * kk + 2 + hp] = pack_bf16(k0 - hk0, k1 - hk1);
        }
      tc::st16x256b<KK>(t_hi, ahi);
      tc::st16x256b<KK>(t_lo, alo);
    }
    tc::wait_st();
    tc::fence_before();
    __syncthreads();
    if (tid == 0) {
      tc::fence_after();
      const int passes = a.state_split ? 3 : 2;  // A_hi S_hi, A_lo S_hi [, A_hi S_lo]
      for (int pass = 0; pass < passes; ++pass)
#pragma unroll
        for (int kk = 0; kk < KK; ++kk)
          tc::mma_bf16_ta(tmem, tmem + DV + (pass == 1 ? DK / 2 : 0) + 8 * kk,
                          tc::smem_desc(s_img + (pass == 2 ? Lt::IMG : 0) + kk * 2 * Lt::KGRP, Lt::KGRP, 128),
                          kIdesc, pass > 0 || kk > 0);
      tc::commit(mbar);
    }
    ok = tc::mbar_wait(mbar, round & 1u, kWait) && ok;
    ++round;
    tc::fence_after();
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
      float acc[NH][4];
      {
        uint32_t r[4 * NH];
        tc::ld16x256b<NH>(t_acc + half * NH * 8, r);
        tc::wait_ld();
#pragma unroll
        for (int j = 0; j < NH; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[j][e] = __uint_as_float(r[4 * j + e]);
      }
#pragma unroll
      for (int j = 0; j < NH; ++j) {
        const int col0 = (half * NH + j) * 8 + tq * 2;
        float2 vp = make_float2(0.f, 0.f);
        if (valid) {
          if constexpr (FUSED) {
            const __nv_bfloat16* base = a.proj + (brow * T) * a.ld_proj;
            vp = conv_pair<Lt::NCH>(sConv, 2 * DK + col0, t, base + 2 * key_dim + hv * DV + col0, a.ld_proj);
            vp = make_float2(bf16r(silu_fast(vp.x)), bf16r(silu_fast(vp.y)));
          } else {
            const int64_t vo = (row * HV + hv) * DV + col0;
            vp = load2_as_float(a.v, vo, a.x_dtype);
          }
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int col = col0 + e;
          const float vx = e ? vp.y : vp.x;
          float skt = At * acc[j][2 + e];
          float o = At * acc[j][e];
#pragma unroll
          for (int s = 0; s < t; ++s) {
            const float ds = sD[(s * kBeamsPerWarp + g) * DV + col];
            skt += Dst[s] * kkd[s] * ds;
            o += Dst[s] * kqd[s] * ds;
          }
          const float d = bt * (vx - skt);
          o += d * kq_self;
          if (t + 1 < T) dcur[col] = d;
          if constexpr (FUSED) {
            const __nv_bfloat16 ob = __float2bfloat16_rn(o);  // gated_delta returns v's dtype
            const float of = __bfloat162float(ob);
            ss += of * of;
            sO[g * DV + col] = ob;
          } else if (valid) {
            store_from_float(a.out, (row * HV + hv) * DV + col, a.out_dtype, o);
          }
        }
      }
    }
    if (t + 1 < T) {  // keep k_t for the later steps' dot products
      float* kst = sK + (t * kBeamsPerWarp + g) * DK;
#pragma unroll
      for (int kk = 0; kk < KK; ++kk)
#pragma unroll
        for (int e = 0; e < 4; ++e) kst[kk * 16 + tq * 2 + (e & 1) + (e >> 1) * 8] = kv[kk][e];
    }
    Dst[t] = 1.f;
    __syncwarp();
    // ---- gated RMSNorm (fused mixer) -------------------------------------------------
    if constexpr (FUSED) {
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      const float inv = 1.0f / sqrtf(ss / float(DV) + a.norm_eps);
      if (valid) {
        const __nv_bfloat16* zp = a.proj + row * a.ld_proj + conv_dim + hv * DV;
        __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(a.out) + row * (int64_t(HV) * DV) + hv * DV;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const int col = j * 8 + tq * 2;
          const __nv_bfloat162 z = *reinterpret_cast<const __nv_bfloat162*>(zp + col);
          const float o0 = __bfloat162float(sO[g * DV + col]), o1 = __bfloat162float(sO[g * DV + col + 1]);
          const float h0 = bf16r(a.norm_weight[col] * bf16r(o0 * inv));
          const float h1 = bf16r(a.norm_weight[col + 1] * bf16r(o1 * inv));
          *reinterpret_cast<__nv_bfloat162*>(op + col) =
              __floats2bfloat162_rn(h0 * silu_f(__low2float(z)), h1 * silu_f(__high2float(z)));
        }
      }
    }
    __syncwarp();
  }
  }  // octets
  if (!ok && lane == 0) atomicOr(a.status, 1u);  // an MMA completion wait timed out
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::tmem_free(tmem, Lt::TCOLS);
  }
}

template <int DK, int DV, bool FUSED, int TMAX>
int launch_gdn(const GdnArgs& a, cudaStream_t stream) {
  using Lt = Layout<DK, DV>;
  const size_t fixed = Lt::state_bytes(a.state_split != 0) + Lt::conv_bytes(FUSED);
  const size_t per_warp = Lt::warp_bytes(a.T);
  int warps = 4;
  while (warps > 1 && fixed + warps * per_warp > 200 * 1024) warps >>= 1;
  const size_t smem = fixed + warps * per_warp;
  auto kern = gdn_replay_kernel<DK, DV, FUSED, TMAX>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
    set_error("gdn replay: cannot reserve %zu bytes of shared memory", smem);
    return KADLLM_ECUDA;
  }
  GdnArgs args = a;
  args.octets_per_warp = a.W >= 64 ? 2 : 1;
  const int beams_per_cta = warps * kBeamsPerWarp * args.octets_per_warp;
  dim3 grid(a.B * a.HV, (a.W + beams_per_cta - 1) / beams_per_cta);
  kern<<<grid, warps * 32, smem, stream>>>(args);
  KB_CHECK_LAUNCH("gdn replay launch");
  return KADLLM_OK;
}

template <int DK, bool FUSED>
int dispatch_steps(const GdnArgs& a, cudaStream_t stream) {
  if (a.T <= 1) return launch_gdn<DK, DK, FUSED, 1>(a, stream);
  if (a.T <= 2) return launch_gdn<DK, DK, FUSED, 2>(a, stream);
  if (a.T <= 4) return launch_gdn<DK, DK, FUSED, 4>(a, stream);
  return launch_gdn<DK, DK, FUSED, 8>(a, stream);
}

template <bool FUSED>
int dispatch_gdn(int dk, int dv, const GdnArgs& a, cudaStream_t stream) {
  if (dk == 128 && dv == 128) return dispatch_steps<128, FUSED>(a, stream);
  if (dk == 64 && dv == 64) return dispatch_steps<64, FUSED>(a, stream);
  if (dk == 32 && dv == 32) return dispatch_steps<32, FUSED>(a, stream);
  set_error("gdn replay: head dims K=%d V=%d must be equal and in {32, 64, 128}", dk, dv);
  return KADLLM_EUNSUPPORTED;
}

int check_common(int64_t B, int64_t W, int64_t T, int64_t H, int64_t HV, int64_t K, int64_t V) {
  KB_REQUIRE(B >= 1 && W >= 1 && T >= 1 && H >= 1 && HV >= 1 && K >= 1 && V >= 1, KADLLM_EINVAL,
             "gdn replay: empty dimensions");
  KB_REQUIRE(HV % H == 0, KADLLM_EINVAL, "gdn replay: HV=%lld not divisible by H=%lld", (long long)HV,
             (long long)H);
  KB_REQUIRE(T <= kTMax, KADLLM_EUNSUPPORTED, "gdn replay: at most %d suffix steps (got %lld)", kTMax,
             (long long)T);
  KB_REQUIRE(B * HV < (1ll << 31) && B * W < (1ll << 31) && (W + 7) / 8 <= 65535, KADLLM_EINVAL,
             "gdn replay: too many rows");
  return KADLLM_OK;
}

}  // namespace
}  // namespace kb

extern "C" int kadllm_gated_delta_replay(const void* q, const void* k, const void* v, int x_dtype,
                                         const void* log_decay, int decay_dtype, const void* beta,
                                         int beta_dtype, const void* state, int state_dtype, void* out,
                                         int64_t batch, int64_t beam_width, int64_t steps, int64_t heads,
                                         int64_t v_heads, int64_t k_dim, int64_t v_dim, float scale,
                                         uint32_t* status, void* stream) {
  using namespace kb;
  if (int rc = check_common(batch, beam_width, steps, heads, v_heads, k_dim, v_dim)) return rc;
  KB_REQUIRE(valid_dtype(x_dtype) && valid_dtype(decay_dtype) && valid_dtype(beta_dtype) &&
                 valid_dtype(state_dtype),
             KADLLM_EDTYPE, "gdn replay: unsupported dtype code");
  KB_REQUIRE(q && k && v && log_decay && beta && state && out && status, KADLLM_EINVAL, "gdn replay: null pointer");
  const uintptr_t pair = uintptr_t(2 * dtype_size(x_dtype)) - 1;  // q / k / v are read as element pairs
  KB_REQUIRE(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) &
              pair) == 0,
             KADLLM_EINVAL, "gdn replay: q / k / v must be aligned to two elements");
  GdnArgs a{};
  a.q = q; a.k = k; a.v = v; a.x_dtype = x_dtype;
  a.g = log_decay; a.g_dtype = decay_dtype; a.beta = beta; a.beta_dtype = beta_dtype;
  a.state = state; a.state_dtype = state_dtype; a.state_split = state_dtype != KADLLM_BF16;
  a.out = out; a.out_dtype = x_dtype; a.status = status;
  a.B = int(batch); a.W = int(beam_width); a.T = int(steps); a.H = int(heads); a.HV = int(v_heads);
  a.scale = scale > 0.f ? scale : 1.0f / sqrtf(float(k_dim));
  return dispatch_gdn<false>(int(k_dim), int(v_dim), a, static_cast<cudaStream_t>(stream));
}

extern "C" int kadllm_gdn_mixer_replay(const void* proj, int64_t ld_proj, const void* conv_state,
                                       int64_t conv_hist, const void* conv_weight, const void* rec_state,
                                       const float* a_log, const float* dt_bias, const float* norm_weight,
                                       float norm_eps, void* out, int64_t batch, int64_t beam_width,
                                       int64_t steps, int64_t heads, int64_t v_heads, int64_t k_dim,
                                       int64_t v_dim, void* records, uint32_t* status, void* stream) {
  using namespace kb;
  if (int rc = check_common(batch, beam_width, steps, heads, v_heads, k_dim, v_dim)) return rc;
  KB_REQUIRE(proj && conv_state && conv_weight && rec_state && a_log && dt_bias && norm_weight && out && status,
             KADLLM_EINVAL, "gdn mixer: null pointer");
  const int64_t conv_dim = 2 * heads * k_dim + v_heads * v_dim;
  KB_REQUIRE(conv_hist >= 3, KADLLM_EINVAL, "gdn mixer: conv state needs >= 3 taps");
  KB_REQUIRE(ld_proj >= conv_dim + v_heads * v_dim + 2 * v_heads && ld_proj % 2 == 0 &&
                 (reinterpret_cast<uintptr_t>(proj) & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 3) == 0,
             KADLLM_EINVAL, "gdn mixer: projection row too short or misaligned");
  GdnArgs a{};
  a.proj = static_cast<const __nv_bfloat16*>(proj); a.ld_proj = ld_proj;
  a.conv_state = static_cast<const __nv_bfloat16*>(conv_state); a.conv_hist = conv_hist;
  a.conv_weight = static_cast<const __nv_bfloat16*>(conv_weight);
  a.a_log = a_log; a.dt_bias = dt_bias; a.norm_weight = norm_weight; a.norm_eps = norm_eps;
  a.state = rec_state; a.state_dtype = KADLLM_BF16; a.state_split = 0;
  a.out = out; a.out_dtype = KADLLM_BF16; a.status = status;
  a.B = int(batch); a.W = int(beam_width); a.T = int(steps); a.H = int(heads); a.HV = int(v_heads);
  a.scale = 1.0f / sqrtf(float(k_dim));
  if (k_dim == v_dim) {
    MixerArgs m{};
    m.proj = a.proj; m.ld_proj = ld_proj; m.conv_state = a.conv_state; m.conv_hist = conv_hist;
    m.conv_weight = a.conv_weight; m.state = static_cast<const __nv_bfloat16*>(rec_state);
    m.a_log = a_log; m.dt_bias = dt_bias; m.norm_weight = norm_weight; m.norm_eps = norm_eps;
    m.out = static_cast<__nv_bfloat16*>(out);
    m.B = a.B; m.W = a.W; m.T = a.T; m.H = a.H; m.HV = a.HV; m.D = int(k_dim); m.scale = a.scale;
    m.status = status;
    m.save = static_cast<unsigned char*>(records);
    if (gdn_mixer_staged_ok(m)) return gdn_mixer_staged(m, static_cast<cudaStream_t>(stream));
  }
  KB_REQUIRE(records == nullptr, KADLLM_EUNSUPPORTED,
             "gdn mixer: first-step records need T = 1, head dims 64 / 128 (K == V) and 16-byte aligned rows");
  return dispatch_gdn<true>(int(k_dim), int(v_dim), a, static_cast<cudaStream_t>(stream));
}

extern "C" int kadllm_gdn_mixer_continue(const void* proj_prev, const int32_t* parent, int64_t prev_width,
                                        const void* proj, int64_t ld_proj, const void* conv_state,
                                        int64_t conv_hist, const void* conv_weight, const void* rec_state,
                                        const float* a_log, const float* dt_bias, const float* norm_weight,
                                        float norm_eps, void* out, int64_t batch, int64_t beam_width,
                                        int64_t heads, int64_t v_heads, int64_t k_dim, int64_t v_dim,
                                        const void* records, uint32_t* status, void* stream) {
  using namespace kb;
  if (int rc = check_common(batch, beam_width, 2, heads, v_heads, k_dim, v_dim)) return rc;
  KB_REQUIRE(proj_prev && parent && proj && conv_state && conv_weight && rec_state && a_log && dt_bias &&
                 norm_weight && out && status,
             KADLLM_EINVAL, "gdn mixer (continuation): null pointer");
  KB_REQUIRE(prev_width >= 1 && prev_width < (int64_t(1) << 30), KADLLM_EINVAL,
             "gdn mixer (continuation): prev_width out of range");
  const int64_t conv_dim = 2 * heads * k_dim + v_heads * v_dim;
  KB_REQUIRE(conv_hist >= 3, KADLLM_EINVAL, "gdn mixer (continuation): conv state needs >= 3 taps");
  KB_REQUIRE(ld_proj >= conv_dim + v_heads * v_dim + 2 * v_heads, KADLLM_EINVAL,
             "gdn mixer (continuation): projection row too short");
  MixerArgs m{};
  m.proj = static_cast<const __nv_bfloat16*>(proj); m.ld_proj = ld_proj;
  m.conv_state = static_cast<const __nv_bfloat16*>(conv_state); m.conv_hist = conv_hist;
  m.conv_weight = static_cast<const __nv_bfloat16*>(conv_weight);
  m.state = static_cast<const __nv_bfloat16*>(rec_state);
  m.a_log = a_log; m.dt_bias = dt_bias; m.norm_weight = norm_weight; m.norm_eps = norm_eps;
  m.out = static_cast<__nv_bfloat16*>(out);
  m.B = int(batch); m.W = int(beam_width); m.T = 2; m.H = int(heads); m.HV = int(v_heads); m.D = int(k_dim);
  m.scale = 1.0f / sqrtf(float(k_dim));
  m.proj_prev = static_cast<const __nv_bfloat16*>(proj_prev); m.parent = parent; m.Wp = int(prev_width);
  m.status = status;
  m.saved = static_cast<const unsigned char*>(records);
  KB_REQUIRE(k_dim == v_dim && gdn_mixer_staged_ok(m), KADLLM_EUNSUPPORTED,
             "gdn mixer (continuation): head dims 64 / 128 (K == V), 16-byte aligned rows only");
  return gdn_mixer_staged(m, static_cast<cudaStream_t>(stream));
}

extern "C" int64_t kadllm_gdn_mixer_record_bytes(int64_t batch, int64_t beam_width, int64_t v_heads, int64_t v_dim) {
  if (batch < 1 || beam_width < 1 || v_heads < 1 || v_dim < 1) return 0;
  return kb::gdn_mixer_record_bytes(batch * beam_width, v_heads, v_dim);
}
