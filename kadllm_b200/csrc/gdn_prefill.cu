// Shared-prefix prefill of the Gated-DeltaNet layers (BF16 activations).
//
// 1. conv_prefill: causal depthwise width-4 conv + SiLU over each request's
//    prompt (zero left padding), and the request's conv state = the last 4
//    pre-conv columns (Transformers Qwen3_5GatedDeltaNet.forward, TF:451-474;
//    the cache keeps F.pad(mixed_qkv, (4 - L, 0)) -> last 4 columns).
// 2. gdn_chunk: the chunked gated delta rule (TF:234-311, chunk 64, UT transform)
//    for one (request, value head) per CTA, with the gates computed from the
//    projection (beta = sigmoid(b), g = -exp(A_log) softplus(a + dt_bias)), q/k
//    L2-normalised in fp32, the output passed through the gated RMSNorm
//    (TF:175-190) and the final recurrent state written once per request in
//    BF16 (the hybrid cache stores it in the conv state's dtype).
//
// Per 64-token chunk c with state S (K x V, fp32 in MMA accumulators):
//     L   = strictly-lower( diag(beta) K K^T  o  exp(G_i - G_j) )
//     T   = (I + L)^-1                                  (blocked fp32 solve)
//     X   = diag(beta) (V - diag(e^G) K S)              (= v_beta - k_cumdecay-part)
//     Vn  = T X                                         (v_new)
//     O   = diag(e^G) Q S + lower( Q K^T o exp(G_i - G_j) ) Vn
//     S  <- e^{G_last} S + K^T diag(e^{G_last - G}) Vn
// All products are bf16 mma.sync tiles with fp32 accumulation; the solve and
// the gate/decay factors are fp32.  TF: transformers/models/qwen3_5/modeling_qwen3_5.py.
#include "mma_tiles.cuh"

namespace kb {
namespace {

// ---------------------------------------------------------------------------
// causal conv1d prefill
// ---------------------------------------------------------------------------
constexpr int kConvTokens = 32;

__global__ void __launch_bounds__(128) conv_prefill_kernel(const __nv_bfloat16* proj, int64_t ld, const __nv_bfloat16* w,
                                                           __nv_bfloat16* out, int64_t ld_out, __nv_bfloat16* state,
                                                           int B, int L, int C) {
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c0 >= C) return;
  const int tiles = (L + kConvTokens - 1) / kConvTokens;
  const int b = blockIdx.y / tiles, tile = blockIdx.y % tiles;
  const int t0 = tile * kConvTokens, t1 = min(L, t0 + kConvTokens);
  float wt[8][4];
#pragma unroll
  for (int e = 0; e < 8; ++e)
#pragma unroll
    for (int j = 0; j < 4; ++j) wt[e][j] = __bfloat162float(w[int64_t(c0 + e) * 4 + j]);
  float win[3][8];
  auto load8 = [&](int t, float (&v)[8]) {
    if (t < 0) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.f;
      return;
    }
    const uint4 u = *reinterpret_cast<const uint4*>(proj + (int64_t(b) * L + t) * ld + c0);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = __low2float(h[j]);
      v[2 * j + 1] = __high2float(h[j]);
    }
  };
  load8(t0 - 3, win[0]);
  load8(t0 - 2, win[1]);
  load8(t0 - 1, win[2]);
  for (int t = t0; t < t1; ++t) {
    float x[8], o[8];
    load8(t, x);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float acc = win[0][e] * wt[e][0] + win[1][e] * wt[e][1] + win[2][e] * wt[e][2] + x[e] * wt[e][3];
      o[e] = silu_f(acc);
      win[0][e] = win[1][e];
      win[1][e] = win[2][e];
      win[2][e] = x[e];
    }
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(o[2 * j], o[2 * j + 1]);
    *reinterpret_cast<uint4*>(out + (int64_t(b) * L + t) * ld_out + c0) = u;
  }
  if (t1 == L) {  // conv state: pre-conv columns L-4 .. L-1 (zeros before the prompt)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      __nv_bfloat16 s4[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = L - 4 + j;
        s4[j] = t >= 0 ? proj[(int64_t(b) * L + t) * ld + c0 + e] : __float2bfloat16_rn(0.f);
      }
      *reinterpret_cast<uint2*>(state + (int64_t(b) * C + c0 + e) * 4) = *reinterpret_cast<uint2*>(s4);
    }
  }
}

// ---------------------------------------------------------------------------
// chunked gated delta rule
// ---------------------------------------------------------------------------
constexpr int kChunk = 64;
constexpr int kThreads = 256;

struct ChunkArgs {
  const __nv_bfloat16* qkv; int64_t ld_qkv;     // [B*L, conv_dim] conv outputs
  const __nv_bfloat16* proj; int64_t ld_proj;   // [B*L, ld] packed projection
  int64_t z_col;                                // first z column in proj (b, a follow z)
  const float* a_log; const float* dt_bias; const float* norm_w; float eps;
  __nv_bfloat16* out; int64_t ld_out;           // [B*L, HV*DV]
  __nv_bfloat16* state;                         // [B, HV, DK, DV]
  int B, L, H, HV;
  float scale;
};

template <int DK, int DV>
struct ChunkSmem {
  static constexpr int SQ = DK + 8, SV = DV + 8, ST = kChunk + 8, SL = kChunk + 1;
  static constexpr size_t q = 0;
  static constexpr size_t k = q + size_t(kChunk) * SQ * 2;
  static constexpr size_t v = k + size_t(kChunk) * SQ * 2;
  static constexpr size_t s = v + size_t(kChunk) * SV * 2;
  static constexpr size_t x = s + size_t(DK) * SV * 2;
  static constexpr size_t vn = x + size_t(kChunk) * SV * 2;
  static constexpr size_t t = vn + size_t(kChunk) * SV * 2;
  static constexpr size_t aqk = t + size_t(kChunk) * ST * 2;
  static constexpr size_t l = aqk + size_t(kChunk) * ST * 2;
  static constexpr size_t tmp = l + size_t(kChunk) * SL * 4;
  static constexpr size_t vec = tmp + size_t(3) * 16 * 16 * 4;
  static constexpr size_t bytes = vec + size_t(kChunk) * 4 * 8;  // G, beta, e^G, e^{GL-G}, ss[2], raw g
};

template <int DK, int DV>
__global__ void __launch_bounds__(kThreads) gdn_chunk_kernel(const ChunkArgs a) {
  using M = ChunkSmem<DK, DV>;
  constexpr int SQ = M::SQ, SV = M::SV, ST = M::ST, SL = M::SL;
  constexpr int KPL = DK / 32, VPL = DV / 32;
  extern __shared__ __align__(16) unsigned char smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem + M::q);
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smem + M::k);
  __nv_bfloat16* sV = reinterpret_cast<__nv_bfloat16*>(smem + M::v);
  __nv_bfloat16* sS = reinterpret_cast<__nv_bfloat16*>(smem + M::s);
  __nv_bfloat16* sX = reinterpret_cast<__nv_bfloat16*>(smem + M::x);
  __nv_bfloat16* sVn = reinterpret_cast<__nv_bfloat16*>(smem + M::vn);
  __nv_bfloat16* sT = reinterpret_cast<__nv_bfloat16*>(smem + M::t);
  __nv_bfloat16* sAqk = reinterpret_cast<__nv_bfloat16*>(smem + M::aqk);
  float* sL = reinterpret_cast<float*>(smem + M::l);
  float* sTmp = reinterpret_cast<float*>(smem + M::tmp);
  float* sG = reinterpret_cast<float*>(smem + M::vec);   // cumulative log decay
  float* sBeta = sG + kChunk;
  float* sEG = sBeta + kChunk;                            // e^{G_i}
  float* sEGL = sEG + kChunk;                             // e^{G_last - G_i}
  float* sSS = sEGL + kChunk;                             // [kChunk][2] partial sum of squares
  float* sRaw = sSS + 2 * kChunk;                         // raw g

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.x / a.HV, hv = blockIdx.x % a.HV;
  const int h = hv / (a.HV / a.H);
  const int key_dim = a.H * DK;
  const int g8 = lane >> 2, tq = lane & 3;

  // state accumulators: warp w owns key rows 16w .. 16w+15 (DK / 16 == 8 warps for DK = 128)
  constexpr int SROWS = DK / 16;  // m-tiles of S
  static_assert(SROWS <= kThreads / 32, "one S m-tile per warp");
  float S[DV / 8][4];
  zero_acc<DV / 8>(S);
  for (int i = tid; i < DK * SV; i += kThreads) sS[i] = __float2bfloat16_rn(0.f);

  const float alog = expf(a.a_log[hv]);
  const float dtb = a.dt_bias[hv];
  const int nchunks = (a.L + kChunk - 1) / kChunk;

  for (int c = 0; c < nchunks; ++c) {
    const int t0 = c * kChunk;
    const int nvalid = min(kChunk, a.L - t0);
    // ---- A: load q, k, v, gates ------------------------------------------------
    for (int i = warp; i < kChunk; i += kThreads / 32) {
      float qv[KPL], kv[KPL], vv[VPL];
      float g = 0.f, beta = 0.f;
      if (i < nvalid) {
        const int64_t row = int64_t(b) * a.L + t0 + i;
        const __nv_bfloat16* src = a.qkv + row * a.ld_qkv;
#pragma unroll
        for (int e = 0; e < KPL; ++e) {
          qv[e] = __bfloat162float(src[h * DK + lane * KPL + e]);
          kv[e] = __bfloat162float(src[key_dim + h * DK + lane * KPL + e]);
        }
#pragma unroll
        for (int e = 0; e < VPL; ++e) vv[e] = __bfloat162float(src[2 * key_dim + hv * DV + lane * VPL + e]);
        const __nv_bfloat16* pr = a.proj + row * a.ld_proj + a.z_col + int64_t(a.HV) * DV;
        beta = bf16r(sigmoid_f(__bfloat162float(pr[hv])));
        g = -alog * softplus_f(__bfloat162float(pr[a.HV + hv]) + dtb);
      } else {
#pragma unroll
        for (int e = 0; e < KPL; ++e) qv[e] = kv[e] = 0.f;
#pragma unroll
        for (int e = 0; e < VPL; ++e) vv[e] = 0.f;
      }
      float sq = 0.f, sk = 0.f;
#pragma unroll
      for (int e = 0; e < KPL; ++e) {
        sq += qv[e] * qv[e];
        sk += kv[e] * kv[e];
      }
      sq = warp_sum(sq);
      sk = warp_sum(sk);
      const float iq = 1.0f / sqrtf(sq + 1e-6f), ik = 1.0f / sqrtf(sk + 1e-6f);
#pragma unroll
      for (int e = 0; e < KPL; ++e) {
        sQ[i * SQ + lane * KPL + e] = __float2bfloat16_rn(qv[e] * iq * a.scale);
        sK[i * SQ + lane * KPL + e] = __float2bfloat16_rn(kv[e] * ik);
      }
#pragma unroll
      for (int e = 0; e < VPL; ++e) sV[i * SV + lane * VPL + e] = __float2bfloat16_rn(vv[e]);
      if (lane == 0) {
        sRaw[i] = g;
        sBeta[i] = beta;
      }
    }
    __syncthreads();
    if (tid == 0) {  // sequential fp32 prefix sum, like torch.cumsum
      float run = 0.f;
      for (int i = 0; i < kChunk; ++i) {
        run += sRaw[i];
        sG[i] = run;
      }
    }
    __syncthreads();
    if (tid < kChunk) {
      sEG[tid] = expf(sG[tid]);
      sEGL[tid] = expf(sG[kChunk - 1] - sG[tid]);
    }
    // ---- B: K K^T -> L (fp32), Q K^T -> Aqk (bf16) ---------------------------------
    {
      const int mt = warp & 3, nh = warp >> 2;
      float kk[4][4], qk[4][4];
      zero_acc<4>(kk);
      zero_acc<4>(qk);
      warp_mma<DK, 4, false, false>(kk, sK, SQ, mt * 16, 0, sK, SQ, 0, nh * 32);
      warp_mma<DK, 4, false, false>(qk, sQ, SQ, mt * 16, 0, sK, SQ, 0, nh * 32);
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = mt * 16 + g8 + (e >> 1) * 8;
          const int col = nh * 32 + j * 8 + tq * 2 + (e & 1);
          const float dec = i >= col ? expf(sG[i] - sG[col]) : 0.f;
          sL[i * SL + col] = i > col ? sBeta[i] * kk[j][e] * dec : 0.f;
          sAqk[i * ST + col] = __float2bfloat16_rn(i >= col ? qk[j][e] * dec : 0.f);
        }
    }
    __syncthreads();
    // ---- C: T = (I + L)^-1 (blocked forward substitution, fp32, in place) ---------
    if (warp < 4) {  // diagonal 16x16 blocks
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
    for (int I = 1; I < 4; ++I) {
      // P_IJ = sum_{M=J}^{I-1} L_IM T_MJ for all J < I  (T_MM has a unit diagonal)
      float pv[3] = {0.f, 0.f, 0.f};
      for (int J = 0; J < I; ++J) {
        const int i = tid >> 4, j = tid & 15;
        float acc = 0.f;
        for (int Mb = J; Mb < I; ++Mb)
          for (int m = 0; m < 16; ++m) {
            const float lim = sL[(I * 16 + i) * SL + Mb * 16 + m];
            const float tmj = (Mb == J) ? (m == j ? 1.f : (m > j ? sL[(Mb * 16 + m) * SL + J * 16 + j] : 0.f))
                                        : sL[(Mb * 16 + m) * SL + J * 16 + j];
            acc += lim * tmj;
          }
        pv[J] = acc;
      }
      __syncthreads();
      for (int J = 0; J < I; ++J) sTmp[J * 256 + tid] = pv[J];
      __syncthreads();
      // T_IJ = -T_II P_IJ
      for (int J = 0; J < I; ++J) {
        const int i = tid >> 4, j = tid & 15;
        float acc = sTmp[J * 256 + i * 16 + j];  // m == i term (unit diagonal)
        for (int m = 0; m < i; ++m) acc += sL[(I * 16 + i) * SL + I * 16 + m] * sTmp[J * 256 + m * 16 + j];
        pv[J] = -acc;
      }
      __syncthreads();
      for (int J = 0; J < I; ++J) sL[(I * 16 + (tid >> 4)) * SL + J * 16 + (tid & 15)] = pv[J];
      __syncthreads();
    }
    for (int i = tid; i < kChunk * kChunk; i += kThreads) {
      const int r = i / kChunk, col = i % kChunk;
      const float v = r > col ? sL[r * SL + col] : (r == col ? 1.f : 0.f);
      sT[r * ST + col] = __float2bfloat16_rn(v);
    }
    __syncthreads();
    // ---- D: X = diag(beta) (V - diag(e^G) K S) -------------------------------------
    {
      const int mt = warp & 3, nh = warp >> 2;
      constexpr int NT = DV / 16;  // half of the columns per warp
      float y[NT][4];
      zero_acc<NT>(y);
      warp_mma<DK, NT, false, true>(y, sK, SQ, mt * 16, 0, sS, SV, 0, nh * (DV / 2));
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = mt * 16 + g8 + (e >> 1) * 8;
          const int col = nh * (DV / 2) + j * 8 + tq * 2 + (e & 1);
          const float xv = sBeta[i] * (__bfloat162float(sV[i * SV + col]) - sEG[i] * y[j][e]);
          sX[i * SV + col] = __float2bfloat16_rn(xv);
        }
    }
    __syncthreads();
    // ---- E: Vn = T X; keep Vn and diag(e^{G_last - G}) Vn -----------------------------
    {
      const int mt = warp & 3, nh = warp >> 2;
      constexpr int NT = DV / 16;
      float vn[NT][4];
      zero_acc<NT>(vn);
      warp_mma<kChunk, NT, false, true>(vn, sT, ST, mt * 16, 0, sX, SV, 0, nh * (DV / 2));
      __syncthreads();
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = mt * 16 + g8 + (e >> 1) * 8;
          const int col = nh * (DV / 2) + j * 8 + tq * 2 + (e & 1);
          sVn[i * SV + col] = __float2bfloat16_rn(vn[j][e]);
          sX[i * SV + col] = __float2bfloat16_rn(vn[j][e] * sEGL[i]);
        }
    }
    __syncthreads();
    // ---- F: O = diag(e^G) Q S + Aqk Vn, gated RMSNorm, store --------------------------
    {
      const int mt = warp & 3, nh = warp >> 2;
      constexpr int NT = DV / 16;
      float o[NT][4];
      zero_acc<NT>(o);
      warp_mma<DK, NT, false, true>(o, sQ, SQ, mt * 16, 0, sS, SV, 0, nh * (DV / 2));
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const float e0 = sEG[mt * 16 + g8], e1 = sEG[mt * 16 + g8 + 8];
        o[j][0] *= e0; o[j][1] *= e0; o[j][2] *= e1; o[j][3] *= e1;
      }
      warp_mma<kChunk, NT, false, true>(o, sAqk, ST, mt * 16, 0, sVn, SV, 0, nh * (DV / 2));
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
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int i = mt * 16 + g8 + half * 8;
        if (i >= nvalid) continue;
        const float var = (sSS[i * 2] + sSS[i * 2 + 1]) / float(DV);
        const float inv = 1.0f / sqrtf(var + a.eps);
        const int64_t row = int64_t(b) * a.L + t0 + i;
        const __nv_bfloat16* zp = a.proj + row * a.ld_proj + a.z_col + hv * DV;
        __nv_bfloat16* op = a.out + row * a.ld_out + hv * DV;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const int col = nh * (DV / 2) + j * 8 + tq * 2;
          const __nv_bfloat162 zz = *reinterpret_cast<const __nv_bfloat162*>(zp + col);
          const float h0 = bf16r(a.norm_w[col] * bf16r(o[j][half * 2] * inv));
          const float h1 = bf16r(a.norm_w[col + 1] * bf16r(o[j][half * 2 + 1] * inv));
          *reinterpret_cast<__nv_bfloat162*>(op + col) =
              __floats2bfloat162_rn(h0 * silu_f(__low2float(zz)), h1 * silu_f(__high2float(zz)));
        }
      }
    }
    __syncthreads();
    // ---- G: S <- e^{G_last} S + K^T (e^{G_last - G} Vn) -------------------------------
    if (warp < SROWS) {
      const float dl = sEG[kChunk - 1];
#pragma unroll
      for (int j = 0; j < DV / 8; ++j) {
        S[j][0] *= dl; S[j][1] *= dl; S[j][2] *= dl; S[j][3] *= dl;
      }
      warp_mma<kChunk, DV / 8, true, true>(S, sK, SQ, warp * 16, 0, sX, SV, 0, 0);
#pragma unroll
      for (int j = 0; j < DV / 8; ++j) {
        const int r0 = warp * 16 + g8, col = j * 8 + tq * 2;
        *reinterpret_cast<__nv_bfloat162*>(sS + r0 * SV + col) = __floats2bfloat162_rn(S[j][0], S[j][1]);
        *reinterpret_cast<__nv_bfloat162*>(sS + (r0 + 8) * SV + col) = __floats2bfloat162_rn(S[j][2], S[j][3]);
      }
    }
    __syncthreads();
  }
  // final state, once per request (BF16, like the hybrid cache)
  if (warp < SROWS) {
    __nv_bfloat16* dst = a.state + (int64_t(b) * a.HV + hv) * DK * DV;
#pragma unroll
    for (int j = 0; j < DV / 8; ++j) {
      const int r0 = warp * 16 + g8, col = j * 8 + tq * 2;
      *reinterpret_cast<__nv_bfloat162*>(dst + r0 * DV + col) = __floats2bfloat162_rn(S[j][0], S[j][1]);
      *reinterpret_cast<__nv_bfloat162*>(dst + (r0 + 8) * DV + col) = __floats2bfloat162_rn(S[j][2], S[j][3]);
    }
  }
}

template <int DK, int DV>
int launch_chunk(const ChunkArgs& a, cudaStream_t s) {
  const size_t smem = ChunkSmem<DK, DV>::bytes;
  auto kern = gdn_chunk_kernel<DK, DV>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
    set_error("gdn prefill: cannot reserve %zu bytes of shared memory", smem);
    return KADLLM_ECUDA;
  }
  kern<<<a.B * a.HV, kThreads, smem, s>>>(a);
  KB_CHECK_LAUNCH("gdn prefill launch");
  return KADLLM_OK;
}

}  // namespace
}  // namespace kb

using namespace kb;

extern "C" int kadllm_conv1d_prefill(const void* proj, int64_t ld_proj, const void* weight, void* out,
                                     int64_t ld_out, void* conv_state, int64_t batch, int64_t length,
                                     int64_t channels, void* stream) {
  KB_REQUIRE(proj && weight && out && conv_state, KADLLM_EINVAL, "conv prefill: null pointer");
  KB_REQUIRE(batch >= 1 && length >= 1 && channels >= 1, KADLLM_EINVAL, "conv prefill: empty");
  KB_REQUIRE(channels % 8 == 0 && ld_proj % 8 == 0 && ld_out % 8 == 0 &&
                 (reinterpret_cast<uintptr_t>(proj) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                 (reinterpret_cast<uintptr_t>(conv_state) & 7) == 0,
             KADLLM_EINVAL, "conv prefill: channels / strides must be multiples of 8 and rows 16-byte aligned");
  const int tiles = int((length + kConvTokens - 1) / kConvTokens);
  KB_REQUIRE(batch * tiles <= 65535, KADLLM_EINVAL, "conv prefill: too many token tiles");
  dim3 grid(unsigned((channels / 8 + 127) / 128), unsigned(batch * tiles));
  conv_prefill_kernel<<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(proj), ld_proj, static_cast<const __nv_bfloat16*>(weight),
      static_cast<__nv_bfloat16*>(out), ld_out, static_cast<__nv_bfloat16*>(conv_state), int(batch), int(length),
      int(channels));
  KB_CHECK_LAUNCH("conv prefill launch");
  return KADLLM_OK;
}

extern "C" int kadllm_gdn_prefill(const void* qkv, int64_t ld_qkv, const void* proj, int64_t ld_proj, int64_t z_col,
                                  const float* a_log, const float* dt_bias, const float* norm_weight, float norm_eps,
                                  void* out, int64_t ld_out, void* state, int64_t batch, int64_t length,
                                  int64_t heads, int64_t v_heads, int64_t k_dim, int64_t v_dim, void* stream) {
  KB_REQUIRE(qkv && proj && a_log && dt_bias && norm_weight && out && state, KADLLM_EINVAL,
             "gdn prefill: null pointer");
  KB_REQUIRE(batch >= 1 && length >= 1 && heads >= 1 && v_heads >= 1 && v_heads % heads == 0, KADLLM_EINVAL,
             "gdn prefill: bad dimensions");
  KB_REQUIRE(ld_out % 2 == 0 && ld_proj % 2 == 0 && z_col % 2 == 0, KADLLM_EINVAL, "gdn prefill: odd strides");
  ChunkArgs a{};
  a.qkv = static_cast<const __nv_bfloat16*>(qkv); a.ld_qkv = ld_qkv;
  a.proj = static_cast<const __nv_bfloat16*>(proj); a.ld_proj = ld_proj; a.z_col = z_col;
  a.a_log = a_log; a.dt_bias = dt_bias; a.norm_w = norm_weight; a.eps = norm_eps;
  a.out = static_cast<__nv_bfloat16*>(out); a.ld_out = ld_out;
  a.state = static_cast<__nv_bfloat16*>(state);
  a.B = int(batch); a.L = int(length); a.H = int(heads); a.HV = int(v_heads);
  a.scale = 1.0f / sqrtf(float(k_dim));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (k_dim == 128 && v_dim == 128) return launch_chunk<128, 128>(a, s);
  if (k_dim == 64 && v_dim == 64) return launch_chunk<64, 64>(a, s);
  if (k_dim == 32 && v_dim == 32) return launch_chunk<32, 32>(a, s);
  set_error("gdn prefill: head dims K=%lld V=%lld must be equal and in {32, 64, 128}", (long long)k_dim,
            (long long)v_dim);
  return KADLLM_EUNSUPPORTED;
}
