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
//     S_{t}^T x = A_t (S0^T x) + sum_{s<=t} D(s,t) d_s (k_s . x),
//     A_t = prod_{r<=t} a_r,  D(s,t) = prod_{s<r<=t} a_r,  a_r = exp(g_r),
// so the only K x V work is the GEMM  P = [q_t ; k_t]_{beams,t} x S0, which runs
// on the tensor cores with S0 staged once in shared memory for all beams of a
// request (a [beams*T*2, K] x [K, V] product per (request, head)).  The fp32
// inputs are split into bf16 hi + lo parts (A = A_hi + A_lo, likewise S0 when
// it is not bf16) so the products keep ~16 mantissa bits; the T-step
// corrections are scalar/vector fp32 work in registers.
//
// One CTA = one (request, value head) pair and a range of beam chunks; a chunk
// holds NB = 32 / T beams so that the GEMM has 64 rows (q and k of NB*T steps).

#include "common.cuh"

namespace kb {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kRows = 64;       // GEMM rows per chunk
constexpr int kBeamSteps = 32;  // NB * T <= 32
constexpr int kTMax = 8;

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
  int state_split;  // 1: state needs a lo part (not bf16)
  void* out;
  int out_dtype;
  int B, W, T, H, HV;
  float scale;
  int NB;
  int chunks_per_cta;
};

template <int DK, int DV>
struct Smem {
  static constexpr int kSStride = DV + 8;   // bf16 elements
  static constexpr int kAStride = DK + 8;   // bf16 elements
  static constexpr int kPStride = DV + 8;   // floats
  static constexpr int kNch = 2 * DK + DV;  // conv channels per CTA (fused)
  static constexpr size_t s_bytes = size_t(DK) * kSStride * 2;
  static constexpr size_t a_bytes = size_t(kRows) * kAStride * 2;
  static constexpr size_t p_bytes = size_t(kRows) * kPStride * 4;
  static constexpr size_t v_bytes = size_t(kBeamSteps) * DV * 4;
  static constexpr size_t coef_floats = 2 * kBeamSteps + 2 * kBeamSteps * kTMax;
  static constexpr size_t conv_bytes = size_t(8) * kNch * 4;
  static size_t total(bool split, bool fused) {
    return s_bytes * (split ? 2 : 1) + 2 * a_bytes + p_bytes + v_bytes + coef_floats * 4 +
           (fused ? conv_bytes : 0);
  }
};

template <int DK, int DV, bool FUSED>
__global__ void __launch_bounds__(kThreads) gdn_replay_kernel(const GdnArgs args) {
  using L = Smem<DK, DV>;
  constexpr int KPL = DK / 32;  // key elements per lane
  constexpr int VPL = DV / 32;  // value elements per lane
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* ptr = smem;
  __nv_bfloat16* sS_hi = reinterpret_cast<__nv_bfloat16*>(ptr);
  ptr += L::s_bytes;
  __nv_bfloat16* sS_lo = nullptr;
  if (args.state_split) {
    sS_lo = reinterpret_cast<__nv_bfloat16*>(ptr);
    ptr += L::s_bytes;
  }
  __nv_bfloat16* sA_hi = reinterpret_cast<__nv_bfloat16*>(ptr);
  ptr += L::a_bytes;
  __nv_bfloat16* sA_lo = reinterpret_cast<__nv_bfloat16*>(ptr);
  ptr += L::a_bytes;
  float* sP = reinterpret_cast<float*>(ptr);
  ptr += L::p_bytes;
  float* sV = reinterpret_cast<float*>(ptr);
  ptr += L::v_bytes;
  float* sDecay = reinterpret_cast<float*>(ptr);  // [kBeamSteps]
  float* sBeta = sDecay + kBeamSteps;             // [kBeamSteps]
  float* sKK = sBeta + kBeamSteps;                // [kBeamSteps * kTMax]
  float* sKQ = sKK + kBeamSteps * kTMax;          // [kBeamSteps * kTMax]
  ptr += L::coef_floats * 4;
  float* sConv = reinterpret_cast<float*>(ptr);  // [8][kNch]: w0..w3, tap0..tap2

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int HV = args.HV, T = args.T, W = args.W;
  const int b = blockIdx.x / HV;
  const int hv = blockIdx.x % HV;
  const int h = hv / (HV / args.H);
  const int key_dim = args.H * DK;
  const int conv_dim = 2 * key_dim + HV * DV;

  // ---- stage S0[b, hv] (K x V) as bf16 hi (+ lo) --------------------------------
  {
    const int64_t base = (int64_t(b) * HV + hv) * DK * DV;
    for (int i = tid * 4; i < DK * DV; i += kThreads * 4) {
      float f[4];
      load4(args.state, base + i, args.state_dtype, f);
      const int kr = i / DV, vc = i % DV;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat16 hi = __float2bfloat16_rn(f[e]);
        sS_hi[kr * L::kSStride + vc + e] = hi;
        if (args.state_split) sS_lo[kr * L::kSStride + vc + e] = __float2bfloat16_rn(f[e] - __bfloat162float(hi));
      }
    }
    for (int i = tid; i < kRows * L::kAStride; i += kThreads) {
      sA_hi[i] = __float2bfloat16_rn(0.f);
      sA_lo[i] = __float2bfloat16_rn(0.f);
    }
    if constexpr (FUSED) {
      for (int c = tid; c < L::kNch; c += kThreads) {
        int ch;
        if (c < DK) ch = h * DK + c;
        else if (c < 2 * DK) ch = key_dim + h * DK + (c - DK);
        else ch = 2 * key_dim + hv * DV + (c - 2 * DK);
        const __nv_bfloat16* w = args.conv_weight + int64_t(ch) * 4;
        const __nv_bfloat16* s = args.conv_state + (int64_t(b) * conv_dim + ch) * args.conv_hist + args.conv_hist - 3;
#pragma unroll
        for (int j = 0; j < 4; ++j) sConv[j * L::kNch + c] = __bfloat162float(w[j]);
#pragma unroll
        for (int j = 0; j < 3; ++j) sConv[(4 + j) * L::kNch + c] = __bfloat162float(s[j]);
      }
    }
  }
  __syncthreads();

  const int NB = args.NB;
  const int chunks_total = (W + NB - 1) / NB;
  const int c_begin = blockIdx.y * args.chunks_per_cta;
  const int c_end = min(chunks_total, c_begin + args.chunks_per_cta);

  for (int chunk = c_begin; chunk < c_end; ++chunk) {
    const int beam0 = chunk * NB;
    const int nb = min(NB, W - beam0);

    // ---- phase 1: q/k/v (conv + SiLU when fused), norms, gates, dot products -----
    for (int n = warp; n < nb; n += kWarps) {
      const int64_t r = int64_t(b) * W + beam0 + n;  // beam row in [0, BW)
      float qn[kTMax][KPL], kn[kTMax][KPL];
      float qwin[3][KPL], kwin[3][KPL], vwin[3][VPL];
      if constexpr (FUSED) {
#pragma unroll
        for (int j = 0; j < 3; ++j) {
#pragma unroll
          for (int e = 0; e < KPL; ++e) {
            qwin[j][e] = sConv[(4 + j) * L::kNch + lane * KPL + e];
            kwin[j][e] = sConv[(4 + j) * L::kNch + DK + lane * KPL + e];
          }
#pragma unroll
          for (int e = 0; e < VPL; ++e) vwin[j][e] = sConv[(4 + j) * L::kNch + 2 * DK + lane * VPL + e];
        }
      }
#pragma unroll
      for (int t = 0; t < kTMax; ++t) {
        if (t < T) {
          const int64_t row = r * T + t;
          float qv[KPL], kv[KPL], vv[VPL];
          float gt, bt;
          if constexpr (FUSED) {
            const __nv_bfloat16* pr = args.proj + row * args.ld_proj;
            // conv over [3 prefix taps, suffix] then SiLU, rounded to bf16 like the
            // conv operator's output (src/kadllm/kernels/causal_conv1d.py:41-48)
#pragma unroll
            for (int e = 0; e < KPL; ++e) {
              const int cq = lane * KPL + e;
              const float xq = __bfloat162float(pr[h * DK + cq]);
              const float xk = __bfloat162float(pr[key_dim + h * DK + cq]);
              float aq = qwin[0][e] * sConv[0 * L::kNch + cq] + qwin[1][e] * sConv[1 * L::kNch + cq] +
                         qwin[2][e] * sConv[2 * L::kNch + cq] + xq * sConv[3 * L::kNch + cq];
              float ak = kwin[0][e] * sConv[0 * L::kNch + DK + cq] + kwin[1][e] * sConv[1 * L::kNch + DK + cq] +
                         kwin[2][e] * sConv[2 * L::kNch + DK + cq] + xk * sConv[3 * L::kNch + DK + cq];
              qv[e] = bf16r(silu_f(aq));
              kv[e] = bf16r(silu_f(ak));
              qwin[0][e] = qwin[1][e]; qwin[1][e] = qwin[2][e]; qwin[2][e] = xq;
              kwin[0][e] = kwin[1][e]; kwin[1][e] = kwin[2][e]; kwin[2][e] = xk;
            }
#pragma unroll
            for (int e = 0; e < VPL; ++e) {
              const int cv = lane * VPL + e;
              const float xv = __bfloat162float(pr[2 * key_dim + hv * DV + cv]);
              float av = vwin[0][e] * sConv[0 * L::kNch + 2 * DK + cv] + vwin[1][e] * sConv[1 * L::kNch + 2 * DK + cv] +
                         vwin[2][e] * sConv[2 * L::kNch + 2 * DK + cv] + xv * sConv[3 * L::kNch + 2 * DK + cv];
              vv[e] = bf16r(silu_f(av));
              vwin[0][e] = vwin[1][e]; vwin[1][e] = vwin[2][e]; vwin[2][e] = xv;
            }
            const int64_t gcol = conv_dim + int64_t(HV) * DV;
            const float bl = __bfloat162float(pr[gcol + hv]);
            const float al = __bfloat162float(pr[gcol + HV + hv]);
            bt = bf16r(sigmoid_f(bl));
            gt = -expf(args.a_log[hv]) * softplus_f(al + args.dt_bias[hv]);
          } else {
            const int64_t qo = (row * args.H + h) * DK + lane * KPL;
            const int64_t vo = (row * HV + hv) * DV + lane * VPL;
#pragma unroll
            for (int e = 0; e < KPL; ++e) {
              qv[e] = load_as_float(args.q, qo + e, args.x_dtype);
              kv[e] = load_as_float(args.k, qo + e, args.x_dtype);
            }
#pragma unroll
            for (int e = 0; e < VPL; ++e) vv[e] = load_as_float(args.v, vo + e, args.x_dtype);
            gt = load_as_float(args.g, row * HV + hv, args.g_dtype);
            bt = load_as_float(args.beta, row * HV + hv, args.beta_dtype);
          }
          float sq = 0.f, sk = 0.f;
#pragma unroll
          for (int e = 0; e < KPL; ++e) {
            sq += qv[e] * qv[e];
            sk += kv[e] * kv[e];
          }
          sq = warp_sum(sq);
          sk = warp_sum(sk);
          const float dq = sqrtf(sq + 1e-6f), dk = sqrtf(sk + 1e-6f);
          const int qrow = n * 2 * T + t, krow = n * 2 * T + T + t;
#pragma unroll
          for (int e = 0; e < KPL; ++e) {
            qn[t][e] = qv[e] / dq * args.scale;
            kn[t][e] = kv[e] / dk;
            const __nv_bfloat16 qh = __float2bfloat16_rn(qn[t][e]);
            const __nv_bfloat16 kh = __float2bfloat16_rn(kn[t][e]);
            sA_hi[qrow * L::kAStride + lane * KPL + e] = qh;
            sA_lo[qrow * L::kAStride + lane * KPL + e] = __float2bfloat16_rn(qn[t][e] - __bfloat162float(qh));
            sA_hi[krow * L::kAStride + lane * KPL + e] = kh;
            sA_lo[krow * L::kAStride + lane * KPL + e] = __float2bfloat16_rn(kn[t][e] - __bfloat162float(kh));
          }
#pragma unroll
          for (int e = 0; e < VPL; ++e) sV[(n * T + t) * DV + lane * VPL + e] = vv[e];
          // dot products against earlier keys: kq[s][t] (s <= t), kk[s][t] (s < t)
#pragma unroll
          for (int s = 0; s < kTMax; ++s) {
            if (s <= t) {
              float dqs = 0.f, dks = 0.f;
#pragma unroll
              for (int e = 0; e < KPL; ++e) {
                dqs += kn[s][e] * qn[t][e];
                dks += kn[s][e] * kn[t][e];
              }
              dqs = warp_sum(dqs);
              dks = warp_sum(dks);
              if (lane == 0) {
                sKQ[(n * T + s) * T + t] = dqs;
                sKK[(n * T + s) * T + t] = dks;
              }
            }
          }
          if (lane == 0) {
            sDecay[n * T + t] = expf(gt);
            sBeta[n * T + t] = bt;
          }
        }
      }
    }
    __syncthreads();

    // ---- phase 2: P = A x S0 on the tensor cores (A = q/k rows, split hi+lo) -------
    {
      const int rows_used = nb * 2 * T;
      constexpr int kNGroups = DV / 32;
      for (int item = warp; item < 4 * kNGroups; item += kWarps) {
        const int mt = item % 4, ng = item / 4;
        if (mt * 16 >= rows_used) continue;
        float acc[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;
        const int passes = args.state_split ? 3 : 2;
        for (int pass = 0; pass < passes; ++pass) {
          const __nv_bfloat16* sa = (pass == 1) ? sA_lo : sA_hi;
          const __nv_bfloat16* ss = (pass == 2) ? sS_lo : sS_hi;
#pragma unroll
          for (int kk = 0; kk < DK / 16; ++kk) {
            uint32_t a[4];
            ldmatrix_x4(a, sa + (mt * 16 + (lane & 15)) * L::kAStride + kk * 16 + (lane >> 4) * 8);
            uint32_t b0[4], b1[4];
            ldmatrix_x4_trans(b0, ss + (kk * 16 + (lane & 15)) * L::kSStride + ng * 32 + (lane >> 4) * 8);
            ldmatrix_x4_trans(b1, ss + (kk * 16 + (lane & 15)) * L::kSStride + ng * 32 + 16 + (lane >> 4) * 8);
            const uint32_t bf0[2] = {b0[0], b0[1]}, bf1[2] = {b0[2], b0[3]};
            const uint32_t bf2[2] = {b1[0], b1[1]}, bf3[2] = {b1[2], b1[3]};
            mma_bf16_16816(acc[0], a, bf0);
            mma_bf16_16816(acc[1], a, bf1);
            mma_bf16_16816(acc[2], a, bf2);
            mma_bf16_16816(acc[3], a, bf3);
          }
        }
        const int g = lane >> 2, tq = lane & 3;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int col = ng * 32 + j * 8 + tq * 2;
          *reinterpret_cast<float2*>(&sP[(mt * 16 + g) * L::kPStride + col]) = make_float2(acc[j][0], acc[j][1]);
          *reinterpret_cast<float2*>(&sP[(mt * 16 + g + 8) * L::kPStride + col]) = make_float2(acc[j][2], acc[j][3]);
        }
      }
    }
    __syncthreads();

    // ---- phase 3: T-step corrections, outputs (+ gated RMSNorm when fused) ---------
    for (int n = warp; n < nb; n += kWarps) {
      const int64_t r = int64_t(b) * W + beam0 + n;
      float delta[kTMax][VPL];
      float D[kTMax];
      float At = 1.f;
#pragma unroll
      for (int t = 0; t < kTMax; ++t) {
        if (t < T) {
          const float a = sDecay[n * T + t];
          const float bt = sBeta[n * T + t];
          At *= a;
#pragma unroll
          for (int s = 0; s < kTMax; ++s)
            if (s < t) D[s] *= a;
          D[t] = 1.f;
          const float* pq = sP + (n * 2 * T + t) * L::kPStride + lane * VPL;
          const float* pk = sP + (n * 2 * T + T + t) * L::kPStride + lane * VPL;
          float o[VPL];
#pragma unroll
          for (int e = 0; e < VPL; ++e) {
            float skt = At * pk[e];
#pragma unroll
            for (int s = 0; s < kTMax; ++s)
              if (s < t) skt += D[s] * sKK[(n * T + s) * T + t] * delta[s][e];
            delta[t][e] = bt * (sV[(n * T + t) * DV + lane * VPL + e] - skt);
            float ov = At * pq[e];
#pragma unroll
            for (int s = 0; s < kTMax; ++s)
              if (s <= t) ov += D[s] * sKQ[(n * T + s) * T + t] * delta[s][e];
            o[e] = ov;
          }
          const int64_t row = r * T + t;
          if constexpr (FUSED) {
            // Qwen3_5RMSNormGated: fp32 normalise, cast, * weight (bf16), * silu(z)
            float ss = 0.f;
#pragma unroll
            for (int e = 0; e < VPL; ++e) {
              o[e] = bf16r(o[e]);
              ss += o[e] * o[e];
            }
            ss = warp_sum(ss);
            const float inv = 1.0f / sqrtf(ss / float(DV) + args.norm_eps);
            const __nv_bfloat16* zp = args.proj + row * args.ld_proj + conv_dim + hv * DV + lane * VPL;
            __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(args.out) + row * (int64_t(HV) * DV) + hv * DV + lane * VPL;
#pragma unroll
            for (int e = 0; e < VPL; ++e) {
              const float hn = bf16r(o[e] * inv);
              const float hw = bf16r(args.norm_weight[lane * VPL + e] * hn);
              const float z = __bfloat162float(zp[e]);
              op[e] = __float2bfloat16_rn(hw * silu_f(z));
            }
          } else {
            const int64_t oo = (row * HV + hv) * DV + lane * VPL;
#pragma unroll
            for (int e = 0; e < VPL; ++e) store_from_float(args.out, oo + e, args.out_dtype, o[e]);
          }
        }
      }
    }
    __syncthreads();
  }
}

template <int DK, int DV, bool FUSED>
int launch_gdn(const GdnArgs& a, cudaStream_t stream) {
  const size_t smem = Smem<DK, DV>::total(a.state_split != 0, FUSED);
  auto kern = gdn_replay_kernel<DK, DV, FUSED>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
    set_error("gdn replay: cannot reserve %zu bytes of shared memory", smem);
    return KADLLM_ECUDA;
  }
  const int pairs = a.B * a.HV;
  const int chunks_total = (a.W + a.NB - 1) / a.NB;
  const int target = 148 * 4;
  int splits = (target + pairs - 1) / pairs;
  splits = splits < 1 ? 1 : (splits > chunks_total ? chunks_total : splits);
  GdnArgs args = a;
  args.chunks_per_cta = (chunks_total + splits - 1) / splits;
  splits = (chunks_total + args.chunks_per_cta - 1) / args.chunks_per_cta;
  dim3 grid(pairs, splits);
  kern<<<grid, kThreads, smem, stream>>>(args);
  KB_CHECK_LAUNCH("gdn replay launch");
  return KADLLM_OK;
}

template <bool FUSED>
int dispatch_gdn(int dk, int dv, const GdnArgs& a, cudaStream_t stream) {
#define KB_GDN_CASE(K_, V_) \
  if (dk == K_ && dv == V_) return launch_gdn<K_, V_, FUSED>(a, stream);
  KB_GDN_CASE(128, 128)
  KB_GDN_CASE(64, 64)
  KB_GDN_CASE(32, 32)
#undef KB_GDN_CASE
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
  KB_REQUIRE(B * HV < (1ll << 31) && B * W < (1ll << 31), KADLLM_EINVAL, "gdn replay: too many rows");
  return KADLLM_OK;
}

}  // namespace
}  // namespace kb

extern "C" int kadllm_gated_delta_replay(const void* q, const void* k, const void* v, int x_dtype,
                                         const void* log_decay, int decay_dtype, const void* beta,
                                         int beta_dtype, const void* state, int state_dtype, void* out,
                                         int64_t batch, int64_t beam_width, int64_t steps, int64_t heads,
                                         int64_t v_heads, int64_t k_dim, int64_t v_dim, float scale,
                                         void* stream) {
  using namespace kb;
  if (int rc = check_common(batch, beam_width, steps, heads, v_heads, k_dim, v_dim)) return rc;
  KB_REQUIRE(valid_dtype(x_dtype) && valid_dtype(decay_dtype) && valid_dtype(beta_dtype) &&
                 valid_dtype(state_dtype),
             KADLLM_EDTYPE, "gdn replay: unsupported dtype code");
  KB_REQUIRE(q && k && v && log_decay && beta && state && out, KADLLM_EINVAL, "gdn replay: null pointer");
  GdnArgs a{};
  a.q = q; a.k = k; a.v = v; a.x_dtype = x_dtype;
  a.g = log_decay; a.g_dtype = decay_dtype; a.beta = beta; a.beta_dtype = beta_dtype;
  a.state = state; a.state_dtype = state_dtype; a.state_split = state_dtype != KADLLM_BF16;
  a.out = out; a.out_dtype = x_dtype;
  a.B = int(batch); a.W = int(beam_width); a.T = int(steps); a.H = int(heads); a.HV = int(v_heads);
  a.scale = scale > 0.f ? scale : 1.0f / sqrtf(float(k_dim));
  a.NB = kBeamSteps / a.T;
  return dispatch_gdn<false>(int(k_dim), int(v_dim), a, static_cast<cudaStream_t>(stream));
}

extern "C" int kadllm_gdn_mixer_replay(const void* proj, int64_t ld_proj, const void* conv_state,
                                       int64_t conv_hist, const void* conv_weight, const void* rec_state,
                                       const float* a_log, const float* dt_bias, const float* norm_weight,
                                       float norm_eps, void* out, int64_t batch, int64_t beam_width,
                                       int64_t steps, int64_t heads, int64_t v_heads, int64_t k_dim,
                                       int64_t v_dim, void* stream) {
  using namespace kb;
  if (int rc = check_common(batch, beam_width, steps, heads, v_heads, k_dim, v_dim)) return rc;
  KB_REQUIRE(proj && conv_state && conv_weight && rec_state && a_log && dt_bias && norm_weight && out,
             KADLLM_EINVAL, "gdn mixer: null pointer");
  const int64_t conv_dim = 2 * heads * k_dim + v_heads * v_dim;
  KB_REQUIRE(conv_hist >= 3, KADLLM_EINVAL, "gdn mixer: conv state needs >= 3 taps");
  KB_REQUIRE(ld_proj >= conv_dim + v_heads * v_dim + 2 * v_heads, KADLLM_EINVAL,
             "gdn mixer: projection row too short");
  GdnArgs a{};
  a.proj = static_cast<const __nv_bfloat16*>(proj); a.ld_proj = ld_proj;
  a.conv_state = static_cast<const __nv_bfloat16*>(conv_state); a.conv_hist = conv_hist;
  a.conv_weight = static_cast<const __nv_bfloat16*>(conv_weight);
  a.a_log = a_log; a.dt_bias = dt_bias; a.norm_weight = norm_weight; a.norm_eps = norm_eps;
  a.state = rec_state; a.state_dtype = KADLLM_BF16; a.state_split = 0;
  a.out = out; a.out_dtype = KADLLM_BF16;
  a.B = int(batch); a.W = int(beam_width); a.T = int(steps); a.H = int(heads); a.HV = int(v_heads);
  a.scale = 1.0f / sqrtf(float(k_dim));
  a.NB = kBeamSteps / a.T;
  return dispatch_gdn<true>(int(k_dim), int(v_dim), a, static_cast<cudaStream_t>(stream));
}
