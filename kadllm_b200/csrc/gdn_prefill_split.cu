// Prompt prefill of the Gated-DeltaNet layers, split into a parallel chunk
// preparation and a lean sequential state scan (BF16 activations, fp32 state).
//
// Semantics: Transformers Qwen3_5GatedDeltaNet.forward on the prompt
// (transformers/models/qwen3_5/modeling_qwen3_5.py:422-533): causal conv1d +
// SiLU (zero left padding), gates beta = sigmoid(b), g = -exp(A_log) softplus(a +
// dt_bias), q/k L2-normalised (here in fp32), the chunked gated delta rule with
// the UT transform (chunk 64, modeling_qwen3_5.py:234-311), the gated RMSNorm
// (modeling_qwen3_5.py:175-190), plus the request-sized prefix the decode
// replays from: the last 4 pre-conv columns and the final recurrent state, BF16
// like the hybrid cache (transformers/cache_utils.py:734-800).
//
// prep  (grid: chunks x B*HV, 4 warps) -- everything that does not depend on the
//       recurrent state, for all chunks at once:
//         conv + SiLU from the projection, normalised q (scaled) / k, v, the
//         in-chunk cumulative decay G and beta, the tensor-core products K K^T
//         and Q K^T, and T = (I + L)^-1 for L = strictly-lower(diag(beta) K K^T o
//         exp(G_i - G_j)) by 16x16 forward substitution and two levels of block
//         merges [[A,0],[C,D]]^-1 = [[A^-1,0],[-D^-1 C A^-1, D^-1]] (fp32).
// scan  (grid: B*HV, 8 warps) -- per chunk, with the next chunk's operands
//       prefetched by cp.async:
//         X  = diag(beta) (V - diag(e^G) K S)        Vn = T X
//         O  = diag(e^G) Q S + Aqk Vn  -> gated RMSNorm -> out
//         S <- e^{G_last} S + K^T diag(e^{G_last - G}) Vn
// S stays in fp32 MMA accumulators; operands are bf16 tensor-core tiles.
#include "mma_tiles.cuh"

namespace kb {
namespace {

constexpr int kC = 64;  // chunk length

struct SplitArgs {
  const __nv_bfloat16* proj; int64_t ld_proj;  // [B*L, ld]: q | k | v | z | b | a
  const __nv_bfloat16* conv_w;                 // [conv_dim, 4]
  __nv_bfloat16* conv_state;                   // [B, conv_dim, 4]
  const float* a_log; const float* dt_bias; const float* norm_w; float eps;
  __nv_bfloat16* out; int64_t ld_out;          // [B*L, HV*DV]
  __nv_bfloat16* state;                        // [B, HV, DK, DV]
  // workspace (per (b, hv), tokens padded to a whole number of chunks)
  __nv_bfloat16* qn;    // [B*HV, Lp, DK]
  __nv_bfloat16* kn;    // [B*HV, Lp, DK]
  __nv_bfloat16* vv;    // [B*HV, Lp, DV]
  __nv_bfloat16* tmat;  // [B*HV, nc, 64, 64]
  __nv_bfloat16* aqk;   // [B*HV, nc, 64, 64]
  float* gcum;          // [B*HV, Lp]
  float* beta;          // [B*HV, Lp]
  int B, L, Lp, nc, H, HV;
  float scale;
};

template <int DK, int DV>
struct WsLayout {
  static size_t bytes(int64_t B, int64_t HV, int64_t L) {
    const int64_t nc = (L + kC - 1) / kC, Lp = nc * kC, n = B * HV;
    return size_t(n) * (Lp * (2 * DK + DV) * 2 + nc * kC * kC * 2 * 2 + Lp * 4 * 2) + 1024;
  }
};

// ---------------------------------------------------------------------------
// prep
// ---------------------------------------------------------------------------
template <int DK, int DV>
struct PrepSmem {
  static constexpr int SQ = DK + 8, SL = kC + 1;
  static constexpr size_t q = 0;
  static constexpr size_t k = q + size_t(kC) * SQ * 2;
  static constexpr size_t l = k + size_t(kC) * SQ * 2;
  static constexpr size_t tmp = l + size_t(kC) * SL * 4;
  static constexpr size_t vec = tmp + size_t(32) * 33 * 4;
  static constexpr size_t bytes = vec + size_t(kC) * 4 * 3;
};

template <int DK, int DV>
__global__ void __launch_bounds__(128) gdn_prep_kernel(const SplitArgs a) {
  using M = PrepSmem<DK, DV>;
  constexpr int SQ = M::SQ, SL = M::SL;
  extern __shared__ __align__(16) unsigned char smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem + M::q);
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smem + M::k);
  float* sL = reinterpret_cast<float*>(smem + M::l);
  float* sTmp = reinterpret_cast<float*>(smem + M::tmp);  // [32][33]
  float* sG = reinterpret_cast<float*>(smem + M::vec);
  float* sBeta = sG + kC;
  float* sRaw = sBeta + kC;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = blockIdx.x;
  const int bh = blockIdx.y, b = bh / a.HV, hv = bh % a.HV, h = hv / (a.HV / a.H);
  const int key_dim = a.H * DK, conv_dim = 2 * key_dim + a.HV * DV;
  const int t0 = c * kC;
  const int64_t tok0 = int64_t(bh) * a.Lp + t0;  // workspace token row of this chunk

  // ---- conv + SiLU for the q / k / v channels of this head (8-channel groups) -------
  constexpr int NG = (2 * DK + DV) / 8;
  constexpr int SEG = 8;  // tokens per work item (plus a 3-token halo)
  for (int item = tid; item < NG * (kC / SEG); item += blockDim.x) {
    const int grp = item % NG, seg = item / NG;
    const int lc = grp * 8;  // local channel: [0, DK) q, [DK, 2DK) k, [2DK, 2DK+DV) v
    const int ch = lc < DK ? h * DK + lc : (lc < 2 * DK ? key_dim + h * DK + (lc - DK) : 2 * key_dim + hv * DV + (lc - 2 * DK));
    float w[8][4];
    {
      const uint4* wp = reinterpret_cast<const uint4*>(a.conv_w + int64_t(ch) * 4);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint4 raw = wp[u];
        const __nv_bfloat162* hw = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          w[2 * u + j][0] = __low2float(hw[2 * j]);
          w[2 * u + j][1] = __high2float(hw[2 * j]);
          w[2 * u + j][2] = __low2float(hw[2 * j + 1]);
          w[2 * u + j][3] = __high2float(hw[2 * j + 1]);
        }
      }
    }
    auto load8 = [&](int t, float (&v)[8]) {
      if (t < 0 || t >= a.L) {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = 0.f;
        return;
      }
      const uint4 u = *reinterpret_cast<const uint4*>(a.proj + (int64_t(b) * a.L + t) * a.ld_proj + ch);
      const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[2 * j] = __low2float(hh[j]);
        v[2 * j + 1] = __high2float(hh[j]);
      }
    };
    const int r0 = seg * SEG;
    float win[3][8];
    load8(t0 + r0 - 3, win[0]);
    load8(t0 + r0 - 2, win[1]);
    load8(t0 + r0 - 1, win[2]);
#pragma unroll 2
    for (int r = r0; r < r0 + SEG; ++r) {
      const int t = t0 + r;
      float x[8], o[8];
      load8(t, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float acc = win[0][e] * w[e][0] + win[1][e] * w[e][1] + win[2][e] * w[e][2] + x[e] * w[e][3];
        o[e] = t < a.L ? silu_fast(acc) : 0.f;
        win[0][e] = win[1][e];
        win[1][e] = win[2][e];
        win[2][e] = x[e];
      }
      uint4 u;
      __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) hh[j] = __floats2bfloat162_rn(o[2 * j], o[2 * j + 1]);
      if (lc < DK) *reinterpret_cast<uint4*>(sQ + r * SQ + lc) = u;
      else if (lc < 2 * DK) *reinterpret_cast<uint4*>(sK + r * SQ + (lc - DK)) = u;
      else *reinterpret_cast<uint4*>(a.vv + (tok0 + r) * DV + (lc - 2 * DK)) = u;
    }
    if (c == a.nc - 1 && seg == kC / SEG - 1) {  // conv state: pre-conv columns L-4 .. L-1
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        __nv_bfloat16 s4[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int t = a.L - 4 + j;
          s4[j] = t >= 0 ? a.proj[(int64_t(b) * a.L + t) * a.ld_proj + ch + e] : __float2bfloat16_rn(0.f);
        }
        *reinterpret_cast<uint2*>(a.conv_state + (int64_t(b) * conv_dim + ch + e) * 4) = *reinterpret_cast<uint2*>(s4);
      }
    }
  }
  // ---- gates ------------------------------------------------------------------------
  if (tid < kC) {
    const int t = t0 + tid;
    float g = 0.f, be = 0.f;
    if (t < a.L) {
      const __nv_bfloat16* pr = a.proj + (int64_t(b) * a.L + t) * a.ld_proj + conv_dim + int64_t(a.HV) * DV;
      be = bf16r(sigmoid_f(__bfloat162float(pr[hv])));
      g = -expf(a.a_log[hv]) * softplus_f(__bfloat162float(pr[a.HV + hv]) + a.dt_bias[hv]);
    }
    sRaw[tid] = g;
    sBeta[tid] = be;
  }
  __syncthreads();
  // ---- L2 normalisation of q (scaled) and k, in place; export --------------------------
  {
    const int r = tid & (kC - 1), part = tid >> 6;  // 128 threads: 64 rows x {q, k}
    __nv_bfloat16* row = (part ? sK : sQ) + r * SQ;
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < DK / 8; ++u) {
      const uint4 raw = *reinterpret_cast<const uint4*>(row + u * 8);
      const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float x0 = __low2float(hh[j]), x1 = __high2float(hh[j]);
        ss += x0 * x0 + x1 * x1;
      }
    }
    const float f = (1.0f / sqrtf(ss + 1e-6f)) * (part ? 1.0f : a.scale);
    __nv_bfloat16* dst = (part ? a.kn : a.qn) + (tok0 + r) * DK;
#pragma unroll
    for (int u = 0; u < DK / 8; ++u) {
      uint4 raw = *reinterpret_cast<const uint4*>(row + u * 8);
      __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) hh[j] = __floats2bfloat162_rn(__low2float(hh[j]) * f, __high2float(hh[j]) * f);
      *reinterpret_cast<uint4*>(row + u * 8) = raw;
      *reinterpret_cast<uint4*>(dst + u * 8) = raw;
    }
  }
  if (warp == 0) {  // in-chunk cumulative log decay (warp scan over 64 values)
    const float v0 = sRaw[2 * lane], v1 = sRaw[2 * lane + 1];
    float run = v0 + v1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, run, o);
      if (lane >= o) run += y;
    }
    const float excl = run - (v0 + v1);
    sG[2 * lane] = excl + v0;
    sG[2 * lane + 1] = excl + v0 + v1;
    a.gcum[tok0 + 2 * lane] = excl + v0;
    a.gcum[tok0 + 2 * lane + 1] = excl + v0 + v1;
    a.beta[tok0 + 2 * lane] = sBeta[2 * lane];
    a.beta[tok0 + 2 * lane + 1] = sBeta[2 * lane + 1];
  }
  __syncthreads();
  // ---- K K^T -> L (fp32), Q K^T -> Aqk (bf16, exported) ------------------------------
  {
    float kk[8][4], qk[8][4];
    zero_acc<8>(kk);
    zero_acc<8>(qk);
    warp_mma<DK, 8, false, false>(kk, sK, SQ, warp * 16, 0, sK, SQ, 0, 0);
    warp_mma<DK, 8, false, false>(qk, sQ, SQ, warp * 16, 0, sK, SQ, 0, 0);
    const int g8 = lane >> 2, tq = lane & 3;
    __nv_bfloat16* aq = a.aqk + (int64_t(bh) * a.nc + c) * kC * kC;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int i = warp * 16 + g8 + hr * 8;
        const int col = j * 8 + tq * 2;
        float av[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int cc = col + e;
          const float dec = i >= cc ? __expf(sG[i] - sG[cc]) : 0.f;
          sL[i * SL + cc] = i > cc ? sBeta[i] * kk[j][hr * 2 + e] * dec : 0.f;
          av[e] = qk[j][hr * 2 + e] * dec;
        }
        *reinterpret_cast<__nv_bfloat162*>(aq + i * kC + col) = __floats2bfloat162_rn(av[0], av[1]);
      }
  }
  __syncthreads();
  // ---- T = (I + L)^-1: diagonal 16x16 blocks by forward substitution ------------------
  {
    const int d0 = warp * 16;
    for (int i = 1; i < 16; ++i) {
      float val = 0.f;
      const int j = lane;
      if (j < i) {
        val = sL[(d0 + i) * SL + d0 + j];
        for (int m = j + 1; m < i; ++m) val += sL[(d0 + i) * SL + d0 + m] * sL[(d0 + m) * SL + d0 + j];
        val = -val;
      }
      __syncwarp();
      if (j < i) sL[(d0 + i) * SL + d0 + j] = val;
      __syncwarp();
    }
  }
  __syncthreads();
  if (tid < kC) sL[tid * SL + tid] = 1.f;  // sL now holds unit-lower blocks (zeros above)
  __syncthreads();
  // level 1 (16x16 blocks, TF32 tensor cores): T_10 = -T_11 (L_10 T_00), T_32 = -T_33 (L_32 T_22)
  {
    const int blk = warp >> 1, nc8 = warp & 1;  // warp -> (block pair, 8-column half)
    const int r0 = 16 + 32 * blk, c0 = 32 * blk;
    float acc[1][4];
    zero_acc<1>(acc);
    warp_mma_tf32<16, 1>(acc, sL + r0 * SL + c0, SL, sL + c0 * SL + c0 + nc8 * 8, SL);
    store_acc<1>(sTmp + blk * 16 * 33 + nc8 * 8, 33, acc, 1.f);
    __syncthreads();
    zero_acc<1>(acc);
    warp_mma_tf32<16, 1>(acc, sL + r0 * SL + r0, SL, sTmp + blk * 16 * 33 + nc8 * 8, 33);
    __syncthreads();
    store_acc<1>(sL + r0 * SL + c0 + nc8 * 8, SL, acc, -1.f);
  }
  __syncthreads();
  // level 2 (32x32 blocks): T_[2:4][0:2] = -T_D (C T_A) with C = L[32:64, 0:32]
  {
    const int mt = warp >> 1, nh = warp & 1;  // 2 m-tiles x 2 column halves of 16
    float acc[2][4];
    zero_acc<2>(acc);
    warp_mma_tf32<32, 2>(acc, sL + (32 + mt * 16) * SL, SL, sL + nh * 16, SL);
    store_acc<2>(sTmp + mt * 16 * 33 + nh * 16, 33, acc, 1.f);
    __syncthreads();
    zero_acc<2>(acc);
    warp_mma_tf32<32, 2>(acc, sL + (32 + mt * 16) * SL + 32, SL, sTmp + nh * 16, 33);
    __syncthreads();
    store_acc<2>(sL + (32 + mt * 16) * SL + nh * 16, SL, acc, -1.f);
  }
  __syncthreads();
  // ---- export T (bf16, unit diagonal) --------------------------------------------------
  {
    __nv_bfloat16* tm = a.tmat + (int64_t(bh) * a.nc + c) * kC * kC;
    for (int e = tid * 2; e < kC * kC; e += blockDim.x * 2) {
      const int i = e / kC, j = e % kC;
      const float v0 = i >= j ? sL[i * SL + j] : 0.f;
      const float v1 = i >= j + 1 ? sL[i * SL + j + 1] : 0.f;
      *reinterpret_cast<__nv_bfloat162*>(tm + e) = __floats2bfloat162_rn(v0, v1);
    }
  }
}

// ---------------------------------------------------------------------------
// scan
// ---------------------------------------------------------------------------
template <int DK, int DV>
struct ScanSmem {
  static constexpr int SQ = DK + 8, SV = DV + 8, ST = kC + 8;
  static constexpr size_t q = 0;
  static constexpr size_t k = q + size_t(kC) * SQ * 2;
  static constexpr size_t v = k + size_t(kC) * SQ * 2;
  static constexpr size_t t = v + size_t(kC) * SV * 2;
  static constexpr size_t aqk = t + size_t(kC) * ST * 2;
  static constexpr size_t g = aqk + size_t(kC) * ST * 2;
  static constexpr size_t be = g + size_t(kC) * 4;
  static constexpr size_t stage = be + size_t(kC) * 4;  // bytes per pipeline stage
  static constexpr size_t s = 2 * stage;
  static constexpr size_t x = s + size_t(DK) * SV * 2;
  static constexpr size_t vn = x + size_t(kC) * SV * 2;
  static constexpr size_t misc = vn + size_t(kC) * SV * 2;  // eG, eGL, ss[2]
  static constexpr size_t bytes = misc + size_t(kC) * 4 * 4;
};

template <int DK, int DV>
__global__ void __launch_bounds__(256) gdn_scan_kernel(const SplitArgs a) {
  using M = ScanSmem<DK, DV>;
  constexpr int SQ = M::SQ, SV = M::SV, ST = M::ST;
  extern __shared__ __align__(16) unsigned char smem[];
  __nv_bfloat16* sS = reinterpret_cast<__nv_bfloat16*>(smem + M::s);
  __nv_bfloat16* sX = reinterpret_cast<__nv_bfloat16*>(smem + M::x);
  __nv_bfloat16* sVn = reinterpret_cast<__nv_bfloat16*>(smem + M::vn);
  float* sEG = reinterpret_cast<float*>(smem + M::misc);
  float* sEGL = sEG + kC;
  float* sSS = sEGL + kC;  // [kC][2]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bh = blockIdx.x, b = bh / a.HV, hv = bh % a.HV;
  const int g8 = lane >> 2, tq = lane & 3;
  const int conv_dim = 2 * a.H * DK + a.HV * DV;

  auto stage_ptr = [&](int st, size_t off) { return smem + st * M::stage + off; };
  auto load_chunk = [&](int c, int st) {
    const int64_t tok0 = int64_t(bh) * a.Lp + int64_t(c) * kC;
    const __nv_bfloat16* gq = a.qn + tok0 * DK;
    const __nv_bfloat16* gk = a.kn + tok0 * DK;
    const __nv_bfloat16* gv = a.vv + tok0 * DV;
    const __nv_bfloat16* gt = a.tmat + (int64_t(bh) * a.nc + c) * kC * kC;
    const __nv_bfloat16* ga = a.aqk + (int64_t(bh) * a.nc + c) * kC * kC;
    __nv_bfloat16* q = reinterpret_cast<__nv_bfloat16*>(stage_ptr(st, M::q));
    __nv_bfloat16* k = reinterpret_cast<__nv_bfloat16*>(stage_ptr(st, M::k));
    __nv_bfloat16* v = reinterpret_cast<__nv_bfloat16*>(stage_ptr(st, M::v));
    __nv_bfloat16* t = reinterpret_cast<__nv_bfloat16*>(stage_ptr(st, M::t));
    __nv_bfloat16* aq = reinterpret_cast<__nv_bfloat16*>(stage_ptr(st, M::aqk));
    for (int i = tid; i < kC * (DK / 8); i += blockDim.x) {
      const int r = i / (DK / 8), cc = (i % (DK / 8)) * 8;
      cp_async16(q + r * SQ + cc, gq + r * DK + cc);
      cp_async16(k + r * SQ + cc, gk + r * DK + cc);
    }
    for (int i = tid; i < kC * (DV / 8); i += blockDim.x) {
      const int r = i / (DV / 8), cc = (i % (DV / 8)) * 8;
      cp_async16(v + r * SV + cc, gv + r * DV + cc);
    }
    for (int i = tid; i < kC * (kC / 8); i += blockDim.x) {
      const int r = i / (kC / 8), cc = (i % (kC / 8)) * 8;
      cp_async16(t + r * ST + cc, gt + r * kC + cc);
      cp_async16(aq + r * ST + cc, ga + r * kC + cc);
    }
    if (tid < kC / 4) {
      cp_async16(stage_ptr(st, M::g) + tid * 16, a.gcum + tok0 + tid * 4);
      cp_async16(stage_ptr(st, M::be) + tid * 16, a.beta + tok0 + tid * 4);
    }
  };

  constexpr int SROWS = DK / 16;
  static_assert(SROWS <= 8, "one S m-tile per warp");
  float S[DV / 8][4];
  zero_acc<DV / 8>(S);
  for (int i = tid; i < DK * SV; i += blockDim.x) sS[i] = __float2bfloat16_rn(0.f);

  load_chunk(0, 0);
  cp_async_commit();
  for (int c = 0; c < a.nc; ++c) {
    const int st = c & 1;
    if (c + 1 < a.nc) {
      load_chunk(c + 1, st ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16* sQ = reinterpret_cast<const __nv_bfloat16*>(stage_ptr(st, M::q));
    const __nv_bfloat16* sK = reinterpret_cast<const __nv_bfloat16*>(stage_ptr(st, M::k));
    const __nv_bfloat16* sV = reinterpret_cast<const __nv_bfloat16*>(stage_ptr(st, M::v));
    const __nv_bfloat16* sT = reinterpret_cast<const __nv_bfloat16*>(stage_ptr(st, M::t));
    const __nv_bfloat16* sA = reinterpret_cast<const __nv_bfloat16*>(stage_ptr(st, M::aqk));
    const float* sG = reinterpret_cast<const float*>(stage_ptr(st, M::g));
    const float* sB = reinterpret_cast<const float*>(stage_ptr(st, M::be));
    if (tid < kC) {
      sEG[tid] = __expf(sG[tid]);
      sEGL[tid] = __expf(sG[kC - 1] - sG[tid]);
    }
    __syncthreads();
    const int mt = warp & 3, nh = warp >> 2;
    constexpr int NT = DV / 16;
    // X = diag(beta) (V - diag(e^G) K S)
    {
      float y[NT][4];
      zero_acc<NT>(y);
      warp_mma<DK, NT, false, true>(y, sK, SQ, mt * 16, 0, sS, SV, 0, nh * (DV / 2));
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int i = mt * 16 + g8 + hr * 8;
          const int col = nh * (DV / 2) + j * 8 + tq * 2;
          const __nv_bfloat162 vv2 = *reinterpret_cast<const __nv_bfloat162*>(sV + i * SV + col);
          const float x0 = sB[i] * (__low2float(vv2) - sEG[i] * y[j][hr * 2]);
          const float x1 = sB[i] * (__high2float(vv2) - sEG[i] * y[j][hr * 2 + 1]);
          *reinterpret_cast<__nv_bfloat162*>(sX + i * SV + col) = __floats2bfloat162_rn(x0, x1);
        }
    }
    __syncthreads();
    // Vn = T X  -> sVn (plain) and sX (scaled by e^{G_last - G}) for the state update
    {
      float vn[NT][4];
      zero_acc<NT>(vn);
      warp_mma<kC, NT, false, true>(vn, sT, ST, mt * 16, 0, sX, SV, 0, nh * (DV / 2));
      __syncthreads();
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int i = mt * 16 + g8 + hr * 8;
          const int col = nh * (DV / 2) + j * 8 + tq * 2;
          *reinterpret_cast<__nv_bfloat162*>(sVn + i * SV + col) = __floats2bfloat162_rn(vn[j][hr * 2], vn[j][hr * 2 + 1]);
          *reinterpret_cast<__nv_bfloat162*>(sX + i * SV + col) =
              __floats2bfloat162_rn(vn[j][hr * 2] * sEGL[i], vn[j][hr * 2 + 1] * sEGL[i]);
        }
    }
    __syncthreads();
    // O = diag(e^G) Q S + Aqk Vn, gated RMSNorm, store
    {
      float o[NT][4];
      zero_acc<NT>(o);
      warp_mma<DK, NT, false, true>(o, sQ, SQ, mt * 16, 0, sS, SV, 0, nh * (DV / 2));
      const float e0 = sEG[mt * 16 + g8], e1 = sEG[mt * 16 + g8 + 8];
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        o[j][0] *= e0; o[j][1] *= e0; o[j][2] *= e1; o[j][3] *= e1;
      }
      warp_mma<kC, NT, false, true>(o, sA, ST, mt * 16, 0, sVn, SV, 0, nh * (DV / 2));
      float ss0 = 0.f, ss1 = 0.f;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) o[j][e] = bf16r(o[j][e]);  // gated_delta output dtype
        ss0 += o[j][0] * o[j][0] + o[j][1] * o[j][1];
        ss1 += o[j][2] * o[j][2] + o[j][3] * o[j][3];
      }
      ss0 += __shfl_xor_sync(0xffffffffu, ss0, 1);
      ss0 += __shfl_xor_sync(0xffffffffu, ss0, 2);
      ss1 += __shfl_xor_sync(0xffffffffu, ss1, 1);
      ss1 += __shfl_xor_sync(0xffffffffu, ss1, 2);
      if (tq == 0) {
        sSS[(mt * 16 + g8) * 2 + nh] = ss0;
        sSS[(mt * 16 + g8 + 8) * 2 + nh] = ss1;
      }
      __syncthreads();
      const int nvalid = min(kC, a.L - c * kC);
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int i = mt * 16 + g8 + hr * 8;
        if (i >= nvalid) continue;
        const float inv = 1.0f / sqrtf((sSS[i * 2] + sSS[i * 2 + 1]) / float(DV) + a.eps);
        const int64_t row = int64_t(b) * a.L + int64_t(c) * kC + i;
        const __nv_bfloat16* zp = a.proj + row * a.ld_proj + conv_dim + hv * DV;
        __nv_bfloat16* op = a.out + row * a.ld_out + hv * DV;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const int col = nh * (DV / 2) + j * 8 + tq * 2;
          const __nv_bfloat162 zz = *reinterpret_cast<const __nv_bfloat162*>(zp + col);
          const float h0 = bf16r(a.norm_w[col] * bf16r(o[j][hr * 2] * inv));
          const float h1 = bf16r(a.norm_w[col + 1] * bf16r(o[j][hr * 2 + 1] * inv));
          *reinterpret_cast<__nv_bfloat162*>(op + col) =
              __floats2bfloat162_rn(h0 * silu_f(__low2float(zz)), h1 * silu_f(__high2float(zz)));
        }
      }
    }
    __syncthreads();
    // S <- e^{G_last} S + K^T (e^{G_last - G} Vn)
    if (warp < SROWS) {
      const float dl = sEG[kC - 1];
#pragma unroll
      for (int j = 0; j < DV / 8; ++j) {
        S[j][0] *= dl; S[j][1] *= dl; S[j][2] *= dl; S[j][3] *= dl;
      }
      warp_mma<kC, DV / 8, true, true>(S, sK, SQ, warp * 16, 0, sX, SV, 0, 0);
#pragma unroll
      for (int j = 0; j < DV / 8; ++j) {
        const int r0 = warp * 16 + g8, col = j * 8 + tq * 2;
        *reinterpret_cast<__nv_bfloat162*>(sS + r0 * SV + col) = __floats2bfloat162_rn(S[j][0], S[j][1]);
        *reinterpret_cast<__nv_bfloat162*>(sS + (r0 + 8) * SV + col) = __floats2bfloat162_rn(S[j][2], S[j][3]);
      }
    }
    __syncthreads();
  }
  if (warp < SROWS) {
    __nv_bfloat16* dst = a.state + int64_t(bh) * DK * DV;
#pragma unroll
    for (int j = 0; j < DV / 8; ++j) {
      const int r0 = warp * 16 + g8, col = j * 8 + tq * 2;
      *reinterpret_cast<__nv_bfloat162*>(dst + r0 * DV + col) = __floats2bfloat162_rn(S[j][0], S[j][1]);
      *reinterpret_cast<__nv_bfloat162*>(dst + (r0 + 8) * DV + col) = __floats2bfloat162_rn(S[j][2], S[j][3]);
    }
  }
}

template <int DK, int DV>
int launch_split(SplitArgs& a, void* ws, int64_t ws_bytes, cudaStream_t s) {
  const int64_t n = int64_t(a.B) * a.HV;
  KB_REQUIRE(ws_bytes >= int64_t(WsLayout<DK, DV>::bytes(a.B, a.HV, a.L)), KADLLM_EINVAL,
             "gdn prefill: workspace too small");
  char* p = static_cast<char*>(ws);
  auto take = [&](size_t bytes) {
    char* r = p;
    p += (bytes + 255) & ~size_t(255);
    return r;
  };
  a.qn = reinterpret_cast<__nv_bfloat16*>(take(size_t(n) * a.Lp * DK * 2));
  a.kn = reinterpret_cast<__nv_bfloat16*>(take(size_t(n) * a.Lp * DK * 2));
  a.vv = reinterpret_cast<__nv_bfloat16*>(take(size_t(n) * a.Lp * DV * 2));
  a.tmat = reinterpret_cast<__nv_bfloat16*>(take(size_t(n) * a.nc * kC * kC * 2));
  a.aqk = reinterpret_cast<__nv_bfloat16*>(take(size_t(n) * a.nc * kC * kC * 2));
  a.gcum = reinterpret_cast<float*>(take(size_t(n) * a.Lp * 4));
  a.beta = reinterpret_cast<float*>(take(size_t(n) * a.Lp * 4));
  if (p - static_cast<char*>(ws) > ws_bytes) {
    set_error("gdn prefill: workspace too small after alignment");
    return KADLLM_EINVAL;
  }
  {
    const size_t smem = PrepSmem<DK, DV>::bytes;
    auto kern = gdn_prep_kernel<DK, DV>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
      set_error("gdn prefill prep: cannot reserve %zu bytes of shared memory", smem);
      return KADLLM_ECUDA;
    }
    kern<<<dim3(a.nc, unsigned(n)), 128, smem, s>>>(a);
    KB_CHECK_LAUNCH("gdn prefill prep launch");
  }
  {
    const size_t smem = ScanSmem<DK, DV>::bytes;
    auto kern = gdn_scan_kernel<DK, DV>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
      set_error("gdn prefill scan: cannot reserve %zu bytes of shared memory", smem);
      return KADLLM_ECUDA;
    }
    kern<<<unsigned(n), 256, smem, s>>>(a);
    KB_CHECK_LAUNCH("gdn prefill scan launch");
  }
  return KADLLM_OK;
}

}  // namespace
}  // namespace kb

using namespace kb;

extern "C" int64_t kadllm_gdn_prefill_workspace(int64_t batch, int64_t length, int64_t v_heads, int64_t k_dim,
                                               int64_t v_dim) {
  if (k_dim == 128 && v_dim == 128) return int64_t(WsLayout<128, 128>::bytes(batch, v_heads, length)) + 8 * 256;
  if (k_dim == 64 && v_dim == 64) return int64_t(WsLayout<64, 64>::bytes(batch, v_heads, length)) + 8 * 256;
  if (k_dim == 32 && v_dim == 32) return int64_t(WsLayout<32, 32>::bytes(batch, v_heads, length)) + 8 * 256;
  return -1;
}

extern "C" int kadllm_gdn_prefill_split(const void* proj, int64_t ld_proj, const void* conv_weight, void* conv_state,
                                        const float* a_log, const float* dt_bias, const float* norm_weight,
                                        float norm_eps, void* out, int64_t ld_out, void* state, void* workspace,
                                        int64_t workspace_bytes, int64_t batch, int64_t length, int64_t heads,
                                        int64_t v_heads, int64_t k_dim, int64_t v_dim, void* stream) {
  KB_REQUIRE(proj && conv_weight && conv_state && a_log && dt_bias && norm_weight && out && state && workspace,
             KADLLM_EINVAL, "gdn prefill: null pointer");
  KB_REQUIRE(batch >= 1 && length >= 1 && heads >= 1 && v_heads >= 1 && v_heads % heads == 0, KADLLM_EINVAL,
             "gdn prefill: bad dimensions");
  KB_REQUIRE(ld_proj % 8 == 0 && ld_out % 2 == 0 && (reinterpret_cast<uintptr_t>(proj) & 15) == 0 &&
                 (reinterpret_cast<uintptr_t>(conv_weight) & 15) == 0 && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0 &&
                 (reinterpret_cast<uintptr_t>(conv_state) & 7) == 0,
             KADLLM_EINVAL, "gdn prefill: projection rows / weights / workspace misaligned");
  const int64_t nc = (length + kC - 1) / kC;
  KB_REQUIRE(nc <= 65535 && batch * v_heads <= 65535, KADLLM_EINVAL, "gdn prefill: grid too large");
  SplitArgs a{};
  a.proj = static_cast<const __nv_bfloat16*>(proj); a.ld_proj = ld_proj;
  a.conv_w = static_cast<const __nv_bfloat16*>(conv_weight);
  a.conv_state = static_cast<__nv_bfloat16*>(conv_state);
  a.a_log = a_log; a.dt_bias = dt_bias; a.norm_w = norm_weight; a.eps = norm_eps;
  a.out = static_cast<__nv_bfloat16*>(out); a.ld_out = ld_out;
  a.state = static_cast<__nv_bfloat16*>(state);
  a.B = int(batch); a.L = int(length); a.nc = int(nc); a.Lp = int(nc * kC); a.H = int(heads); a.HV = int(v_heads);
  a.scale = 1.0f / sqrtf(float(k_dim));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (k_dim == 128 && v_dim == 128) return launch_split<128, 128>(a, workspace, workspace_bytes, s);
  if (k_dim == 64 && v_dim == 64) return launch_split<64, 64>(a, workspace, workspace_bytes, s);
  if (k_dim == 32 && v_dim == 32) return launch_split<32, 32>(a, workspace, workspace_bytes, s);
  set_error("gdn prefill: head dims K=%lld V=%lld must be equal and in {32, 64, 128}", (long long)k_dim,
            (long long)v_dim);
  return KADLLM_EUNSUPPORTED;
}
