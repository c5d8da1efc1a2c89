// Staged GDN decode mixer: causal conv1d replay + SiLU, gates, gated-delta
// replay from the request's shared state and the gated RMSNorm for one
// (request, v-head) per CTA; the fast path of kadllm_gdn_mixer_replay for head
// dims 64 / 128 and one or two suffix tokens (the GRBeam decode steps).
//
// Semantics are those of the general replay kernel (gdn_replay.cu):
// src/kadllm/ops.py:139-163 (gated_delta), :215-226 (causal_conv1d),
// src/kadllm/adapters/qwen3_5.py:144-177 (the mixer) and transformers
// modeling_qwen3_5.py:175-190 (RMSNormGated).  Every beam starts from the same
// state S0 = state[b, hv]; with a_t = exp(g_t), A_t = prod_{r<=t} a_r:
//     S_t^T k_t (before the update) = A_t S0^T k_t + a_t (k_0.k_t) d_0   (t = 1)
//     d_t = beta_t (v_t - that),   o_t = A_t S0^T q_t + [t=1] a_1 (k_0.q_1) d_0 + d_t (k_t.q_t)
// so the only D x D work is [q_t ; k_t] x S0 on the tensor cores.
//
// Data movement: each warp owns beam octets and stages one octet's projection
// slices (the q, k, v, z head slices and the two gate words of all T tokens)
// in shared memory with 16-byte cp.async copies, one octet ahead of the octet
// it computes.  S0 is staged once per CTA with an XOR swizzle that keeps the
// ldmatrix reads conflict-free.  The output tile goes back through the staged
// q slice and leaves as 16-byte stores.
//
// Operand order: the m16n8k16 A fragment of thread (g, tq) holds k columns
// {2tq, 2tq+1, 2tq+8, 2tq+9} of a k16 step.  The contraction order is free, so
// k16 steps 2m and 2m+1 take physical columns 32m + 8tq + [0, 8): a thread's A
// data for two steps is one 16-byte chunk of its staged row, and the ldmatrix
// row addresses of S0 apply the same permutation.  A is split into bf16 hi + lo
// parts (two MMAs), keeping ~16 mantissa bits of the fp32 normalised q and k.
#include "gdn_mixer.cuh"

namespace kb {
namespace {

constexpr int kMixWarps = 4;

template <int D>
struct MixLayout {
  static constexpr int CH = D / 8;          // 16-byte chunks in a head row
  static constexpr int NCH = 3 * D;         // conv channels: q head, k head, v head
  static constexpr int ROWB = 8 * D + 16;   // staged bytes per (token, beam): q, k, v, z, gate words
  static constexpr int S0B = D * D * 2;     // swizzled bf16 state
  static constexpr int TABB = 8 * NCH * 4;  // conv table [8][NCH] fp32
  static constexpr int NWB = D * 4;         // norm weight fp32
  __host__ __device__ static constexpr int octet_bytes(int T) { return T * 8 * ROWB; }
  static size_t smem(int T) { return size_t(S0B) + TABB + NWB + size_t(kMixWarps) * 2 * octet_bytes(T); }
};

// 16-byte chunk swizzle of state row r: distinct over the 8 rows that one
// ldmatrix matrix reads under the permuted k order (bit 0 and bits 3-4 of r).
__device__ __forceinline__ int s0_swz(int r) { return (r & 1) | (((r >> 3) & 3) << 1); }

// cp.async with zero fill when `valid` is false (no bytes read from gmem).
__device__ __forceinline__ void cp16z(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void cp4z(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 4 : 0));
}

__device__ __forceinline__ float2 lo2(float4 v) { return make_float2(v.x, v.y); }
__device__ __forceinline__ float2 hi2(float4 v) { return make_float2(v.z, v.w); }

// Conv + SiLU of 8 consecutive local channels lc (a multiple of 8) at suffix
// step t, rounded to bf16 pairs.  Conv table rows: 0..2 prefix-tap partial
// sums c_t, 3..6 the taps w0..w3; raw input x_s is at byte `xoff` of staged row
// (s, g) (`row0` = row (0, g), rows of one token are 8 * ROWB apart).
template <int NCH, int ROWB>
__device__ __forceinline__ void conv8_silu(const float* tab, int lc, int t, const unsigned char* row0, int xoff,
                                           uint32_t out[4]) {
  float2 acc[4];
  if (t < 3) {
    const float4 c0 = *reinterpret_cast<const float4*>(tab + t * NCH + lc);
    const float4 c1 = *reinterpret_cast<const float4*>(tab + t * NCH + lc + 4);
    acc[0] = lo2(c0); acc[1] = hi2(c0); acc[2] = lo2(c1); acc[3] = hi2(c1);
  } else {
#pragma unroll
    for (int p = 0; p < 4; ++p) acc[p] = make_float2(0.f, 0.f);
  }
#pragma unroll
  for (int s = (t > 3 ? t - 3 : 0); s <= t; ++s) {
    const uint4 x = *reinterpret_cast<const uint4*>(row0 + s * 8 * ROWB + xoff);
    const float* w = tab + (6 - (t - s)) * NCH + lc;
    const float4 w0 = *reinterpret_cast<const float4*>(w), w1 = *reinterpret_cast<const float4*>(w + 4);
    acc[0] = fma2(lo2(w0), bf2f(x.x), acc[0]);
    acc[1] = fma2(hi2(w0), bf2f(x.y), acc[1]);
    acc[2] = fma2(lo2(w1), bf2f(x.z), acc[2]);
    acc[3] = fma2(hi2(w1), bf2f(x.w), acc[3]);
  }
#pragma unroll
  for (int p = 0; p < 4; ++p) out[p] = bf2_pack_f2(silu2(acc[p]));
}

// Same for one channel pair (lc even), returned as the exact bf16 values.
template <int NCH, int ROWB>
__device__ __forceinline__ float2 conv2_silu(const float* tab, int lc, int t, const unsigned char* row0, int xoff) {
  float2 acc = t < 3 ? *reinterpret_cast<const float2*>(tab + t * NCH + lc) : make_float2(0.f, 0.f);
#pragma unroll
  for (int s = (t > 3 ? t - 3 : 0); s <= t; ++s) {
    const uint32_t x = *reinterpret_cast<const uint32_t*>(row0 + s * 8 * ROWB + xoff);
    acc = fma2(*reinterpret_cast<const float2*>(tab + (6 - (t - s)) * NCH + lc), bf2f(x), acc);
  }
  return bf2f(bf2_pack_f2(silu2(acc)));
}

__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v + __shfl_xor_sync(0xffffffffu, v, 2);
}

// Dot product of two threads' bf16 chunks (KM chunks of 8), summed over the quad.
template <int KM>
__device__ __forceinline__ float chunk_dot(const uint32_t (&x)[KM][4], const uint32_t (&y)[KM][4]) {
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int m = 0; m < KM; ++m)
#pragma unroll
    for (int p = 0; p < 4; ++p) acc = fma2(bf2f(x[m][p]), bf2f(y[m][p]), acc);
  return quad_sum(acc.x + acc.y);
}

template <int D, int TMAX>
__global__ void __launch_bounds__(kMixWarps * 32) gdn_mixer_kernel(const MixerArgs a, int octets_per_warp) {
  using L = MixLayout<D>;
  constexpr int CH = L::CH, NCH = L::NCH, ROWB = L::ROWB;
  constexpr int NT = D / 8;   // n8 tiles of the V columns
  constexpr int NH = NT / 2;  // n8 tiles per half (bounds the accumulator registers)
  constexpr int KM = D / 32;  // 16-byte chunks per thread per head row (= k16 step pairs)
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* sS0 = smem;
  float* sTab = reinterpret_cast<float*>(smem + L::S0B);
  float* sNw = sTab + 8 * NCH;
  unsigned char* sStage = smem + L::S0B + L::TABB + L::NWB;

  const int T = a.T;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int HV = a.HV;
  const int b = blockIdx.x / HV, hv = blockIdx.x % HV;
  const int h = hv / (HV / a.H);
  const int key_dim = a.H * D;
  const int conv_dim = 2 * key_dim + HV * D;
  const int64_t ld = a.ld_proj;
  const int octets = (a.W + 7) / 8;
  const int oct0 = (blockIdx.y * kMixWarps + warp) * octets_per_warp;
  const int noct = max(0, min(octets_per_warp, octets - oct0));
  const int obytes = L::octet_bytes(T);
  unsigned char* wbuf = sStage + warp * 2 * obytes;
  // projection columns of the staged slices: q, k, v, z head slices; b and a gate words (aligned down)
  const int col_q = h * D, col_k = key_dim + h * D, col_v = 2 * key_dim + hv * D, col_z = conv_dim + hv * D;
  const int col_b = conv_dim + HV * D + hv, col_a = conv_dim + HV * D + HV + hv;

  // Stage octet `oct` (all T tokens of its 8 beams) into `buf` (one cp.async group per call site).
  auto stage = [&](int oct, unsigned char* buf) {
    const int rows = T * 8;
    for (int idx = lane; idx < rows * 4 * CH; idx += 32) {
      const int r = idx / (4 * CH), piece = (idx / CH) & 3, c = idx % CH;
      const int beam = oct * 8 + (r & 7);
      const bool ok = beam < a.W;
      const int64_t prow = (int64_t(b) * a.W + (ok ? beam : 0)) * T + (r >> 3);
      const int col = piece < 2 ? (piece == 0 ? col_q : col_k) : (piece == 2 ? col_v : col_z);
      cp16z(buf + r * ROWB + piece * 2 * D + c * 16, a.proj + prow * ld + col + c * 8, ok);
    }
    if (lane < rows * 2) {
      const int r = lane >> 1, which = lane & 1;
      const int beam = oct * 8 + (r & 7);
      const bool ok = beam < a.W;
      const int64_t prow = (int64_t(b) * a.W + (ok ? beam : 0)) * T + (r >> 3);
      cp4z(buf + r * ROWB + 8 * D + which * 4, a.proj + prow * ld + ((which ? col_a : col_b) & ~1), ok);
    }
  };

  // ---- CTA prologue: S0 (swizzled), this warp's first octet, conv table, norm weight ----
  {
    const __nv_bfloat16* s0 = a.state + (int64_t(b) * HV + hv) * D * D;
    for (int idx = tid; idx < D * CH; idx += blockDim.x) {
      const int r = idx / CH, c = idx % CH;
      cp_async16(sS0 + r * 2 * D + ((c ^ s0_swz(r)) << 4), s0 + r * D + c * 8);
    }
    cp_async_commit();
  }
  if (noct > 0) stage(oct0, wbuf);
  cp_async_commit();
  for (int c = tid; c < NCH; c += blockDim.x) {
    int ch;
    if (c < D) ch = h * D + c;
    else if (c < 2 * D) ch = key_dim + h * D + (c - D);
    else ch = 2 * key_dim + hv * D + (c - 2 * D);
    const __nv_bfloat16* w = a.conv_weight + int64_t(ch) * 4;
    const __nv_bfloat16* s = a.conv_state + (int64_t(b) * conv_dim + ch) * a.conv_hist + a.conv_hist - 3;
    const float w0 = __bfloat162float(w[0]), w1 = __bfloat162float(w[1]);
    const float w2 = __bfloat162float(w[2]), w3 = __bfloat162float(w[3]);
    const float s0 = __bfloat162float(s[0]), s1 = __bfloat162float(s[1]), s2 = __bfloat162float(s[2]);
    sTab[0 * NCH + c] = w0 * s0 + w1 * s1 + w2 * s2;
    sTab[1 * NCH + c] = w0 * s1 + w1 * s2;
    sTab[2 * NCH + c] = w0 * s2;
    sTab[3 * NCH + c] = w0;  // tap applied to x_{t-3}
    sTab[4 * NCH + c] = w1;
    sTab[5 * NCH + c] = w2;
    sTab[6 * NCH + c] = w3;  // tap applied to x_t
    sTab[7 * NCH + c] = 0.f;
  }
  for (int i = tid; i < D; i += blockDim.x) sNw[i] = a.norm_weight[i];
  const float neg_a = -expf(a.a_log[hv]), dtb = a.dt_bias[hv];
  cp_async_wait<1>();  // S0 landed (the octet copies may still be in flight)
  __syncthreads();

  // ldmatrix row offsets of this lane under the permuted k order, per k16 step parity
  int rowoff[2], swz[2];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int j = lane & 15;
    rowoff[hh] = 8 * ((j & 7) >> 1) + 4 * hh + 2 * (j >> 3) + (j & 1);
    swz[hh] = s0_swz(rowoff[hh]);  // s0_swz(32m + r) == s0_swz(r)
  }

  for (int it = 0; it < noct; ++it) {
    unsigned char* buf = wbuf + (it & 1) * obytes;
    if (it + 1 < noct) stage(oct0 + it + 1, wbuf + ((it + 1) & 1) * obytes);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();

    const unsigned char* row0 = buf + g * ROWB;  // staged row (t = 0, beam g)

    // ---- q_t, k_t (conv + SiLU, bf16), their norms, the gates ----------------------
    uint32_t qw[TMAX][KM][4], kw[TMAX][KM][4];
    float iq[TMAX], ik[TMAX], bt[TMAX], at[TMAX];
#pragma unroll
    for (int t = 0; t < TMAX; ++t) {
      if (t >= T) break;
      float2 sq = make_float2(0.f, 0.f), sk = make_float2(0.f, 0.f);
#pragma unroll
      for (int m = 0; m < KM; ++m) {
        const int c = 4 * m + tq;
        conv8_silu<NCH, ROWB>(sTab, 8 * c, t, row0, c * 16, qw[t][m]);
        conv8_silu<NCH, ROWB>(sTab, D + 8 * c, t, row0, 2 * D + c * 16, kw[t][m]);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float2 qf = bf2f(qw[t][m][p]), kf = bf2f(kw[t][m][p]);
          sq = fma2(qf, qf, sq);
          sk = fma2(kf, kf, sk);
        }
      }
      iq[t] = 1.0f / sqrtf(quad_sum(sq.x + sq.y) + 1e-6f);
      ik[t] = 1.0f / sqrtf(quad_sum(sk.x + sk.y) + 1e-6f);
      const unsigned char* gw = row0 + t * 8 * ROWB + 8 * D;
      const __nv_bfloat162 bw = *reinterpret_cast<const __nv_bfloat162*>(gw);
      const __nv_bfloat162 aw = *reinterpret_cast<const __nv_bfloat162*>(gw + 4);
      const float bv = __bfloat162float((col_b & 1) ? bw.y : bw.x);
      const float av = __bfloat162float((col_a & 1) ? aw.y : aw.x);
      bt[t] = bf16r(sigmoid_f(bv));
      at[t] = expf(neg_a * softplus_f(av + dtb));
    }
    // dot products of the normalised vectors (q also scaled): k_s.q_t (s <= t), k_0.k_1
    float kq[TMAX][TMAX], kk01 = 0.f;
#pragma unroll
    for (int t = 0; t < TMAX; ++t) {
      if (t >= T) break;
#pragma unroll
      for (int s = 0; s <= t; ++s) kq[s][t] = chunk_dot<KM>(kw[s], qw[t]) * ik[s] * iq[t] * a.scale;
      if (t == 1) kk01 = chunk_dot<KM>(kw[0], kw[1]) * ik[0] * ik[1];
    }

    // ---- per token: [q_t ; k_t] x S0 on the tensor cores, recurrence, gated norm ------
    float dreg[TMAX > 1 ? 2 * NT : 1];  // d_0 at this thread's columns (T = 2)
    float At = 1.f;
#pragma unroll
    for (int t = 0; t < TMAX; ++t) {
      if (t >= T) break;
      At *= at[t];
      const float qs = iq[t] * a.scale, ks = ik[t];
      uint32_t ob[NT];
      float ss = 0.f;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float acc[NH][4];
#pragma unroll
        for (int j = 0; j < NH; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll
        for (int m = 0; m < KM; ++m) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            // A rows: g = q_t of beam g, g + 8 = k_t of beam g; hi + lo bf16 parts
            const float2 q0 = mul2(bf2f(qw[t][m][2 * hh]), make_float2(qs, qs));
            const float2 q1 = mul2(bf2f(qw[t][m][2 * hh + 1]), make_float2(qs, qs));
            const float2 k0 = mul2(bf2f(kw[t][m][2 * hh]), make_float2(ks, ks));
            const float2 k1 = mul2(bf2f(kw[t][m][2 * hh + 1]), make_float2(ks, ks));
            uint32_t ahi[4], alo[4];
            ahi[0] = bf2_pack_f2(q0);
            ahi[1] = bf2_pack_f2(k0);
            ahi[2] = bf2_pack_f2(q1);
            ahi[3] = bf2_pack_f2(k1);
            alo[0] = bf2_pack_f2(add2(q0, mul2(bf2f(ahi[0]), make_float2(-1.f, -1.f))));
            alo[1] = bf2_pack_f2(add2(k0, mul2(bf2f(ahi[1]), make_float2(-1.f, -1.f))));
            alo[2] = bf2_pack_f2(add2(q1, mul2(bf2f(ahi[2]), make_float2(-1.f, -1.f))));
            alo[3] = bf2_pack_f2(add2(k1, mul2(bf2f(ahi[3]), make_float2(-1.f, -1.f))));
            const unsigned char* brow = sS0 + (32 * m + rowoff[hh]) * 2 * D;
#pragma unroll
            for (int np = 0; np < NH / 2; ++np) {
              const int chunk = hf * NH + 2 * np + (lane >> 4);
              uint32_t bfr[4];
              ldmatrix_x4_trans(bfr, brow + ((chunk ^ swz[hh]) << 4));
              const uint32_t b0[2] = {bfr[0], bfr[1]}, b1[2] = {bfr[2], bfr[3]};
              mma_bf16_16816(acc[2 * np], ahi, b0);
              mma_bf16_16816(acc[2 * np + 1], ahi, b1);
              mma_bf16_16816(acc[2 * np], alo, b0);
              mma_bf16_16816(acc[2 * np + 1], alo, b1);
            }
          }
        }
        // recurrence at columns (jj*8 + 2tq, +1): acc[j][0..1] = S0^T q_t, acc[j][2..3] = S0^T k_t
#pragma unroll
        for (int j = 0; j < NH; ++j) {
          const int jj = hf * NH + j, col0 = jj * 8 + 2 * tq;
          const float2 vx = conv2_silu<NCH, ROWB>(sTab, 2 * D + col0, t, row0, 4 * D + col0 * 2);
          float2 skt = make_float2(At * acc[j][2], At * acc[j][3]);
          float2 o = make_float2(At * acc[j][0], At * acc[j][1]);
          if (TMAX > 1 && t == 1) {
            const float2 d0 = make_float2(dreg[2 * jj], dreg[2 * jj + 1]);
            skt = fma2(make_float2(at[1] * kk01, at[1] * kk01), d0, skt);
            o = fma2(make_float2(at[1] * kq[0][1], at[1] * kq[0][1]), d0, o);
          }
          const float2 d = mul2(make_float2(bt[t], bt[t]), add2(vx, mul2(skt, make_float2(-1.f, -1.f))));
          o = fma2(d, make_float2(kq[t][t], kq[t][t]), o);
          if (TMAX > 1 && t == 0) {
            dreg[2 * jj] = d.x;
            dreg[2 * jj + 1] = d.y;
          }
          ob[jj] = bf2_pack_f2(o);  // gated_delta returns v's dtype
          const float2 of = bf2f(ob[jj]);
          ss = fmaf(of.x, of.x, fmaf(of.y, of.y, ss));
        }
      }
      // ---- gated RMSNorm, written over this token's staged q slice ---------------------
      const float inv = 1.0f / sqrtf(quad_sum(ss) / float(D) + a.norm_eps);
      unsigned char* rowt = buf + (t * 8 + g) * ROWB;
#pragma unroll
      for (int jj = 0; jj < NT; ++jj) {
        const int col = jj * 8 + 2 * tq;
        const float2 of = bf2f(ob[jj]);
        const float2 z = bf2f(*reinterpret_cast<const uint32_t*>(rowt + 6 * D + col * 2));
        const float2 w = *reinterpret_cast<const float2*>(sNw + col);
        const float2 sz = silu2(z);
        const float h0 = bf16r(w.x * bf16r(of.x * inv)), h1 = bf16r(w.y * bf16r(of.y * inv));
        *reinterpret_cast<uint32_t*>(rowt + col * 2) = bf2_pack(h0 * sz.x, h1 * sz.y);
      }
    }
    __syncwarp();
    // ---- the octet's output rows, 16 bytes per store ------------------------------------
    for (int idx = lane; idx < T * 8 * CH; idx += 32) {
      const int r = idx / CH, c = idx % CH;
      const int ob_beam = (oct0 + it) * 8 + (r & 7);
      if (ob_beam < a.W) {
        const int64_t orow = (int64_t(b) * a.W + ob_beam) * T + (r >> 3);
        *reinterpret_cast<uint4*>(a.out + orow * (int64_t(HV) * D) + hv * D + c * 8) =
            *reinterpret_cast<const uint4*>(buf + r * ROWB + c * 16);
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();
}

template <int D, int TMAX>
int launch_mixer(const MixerArgs& a, cudaStream_t stream) {
  const size_t smem = MixLayout<D>::smem(a.T);
  auto kern = gdn_mixer_kernel<D, TMAX>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
    set_error("gdn mixer: cannot reserve %zu bytes of shared memory", smem);
    return KADLLM_ECUDA;
  }
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int octets = (a.W + 7) / 8;
  const int per_sm = smem * 2 <= 220 * 1024 ? 2 : 1;
  // split a head's octets over enough CTAs to fill about two waves, each warp taking a run of octets
  const int heads = a.B * a.HV;
  int ny = (2 * sms * per_sm + heads - 1) / heads;
  ny = max(1, min(ny, (octets + kMixWarps - 1) / kMixWarps));
  const int opw = (octets + kMixWarps * ny - 1) / (kMixWarps * ny);
  ny = (octets + kMixWarps * opw - 1) / (kMixWarps * opw);
  const dim3 grid{unsigned(heads), unsigned(ny)};
  kern<<<grid, kMixWarps * 32, smem, stream>>>(a, opw);
  KB_CHECK_LAUNCH("gdn mixer launch");
  return KADLLM_OK;
}

}  // namespace

bool gdn_mixer_staged_ok(const MixerArgs& a) {
  if (!(a.D == 64 || a.D == 128) || a.T < 1 || a.T > 2 || a.conv_hist < 3) return false;
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return al16(a.proj) && al16(a.out) && al16(a.state) && a.ld_proj % 8 == 0;
}

int gdn_mixer_staged(const MixerArgs& a, cudaStream_t stream) {
  if (a.D == 128) return a.T == 1 ? launch_mixer<128, 1>(a, stream) : launch_mixer<128, 2>(a, stream);
  return a.T == 1 ? launch_mixer<64, 1>(a, stream) : launch_mixer<64, 2>(a, stream);
}

}  // namespace kb
