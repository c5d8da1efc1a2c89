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
// so the only D x D work is [q_t ; k_t] x S0, on the 5th-generation tensor cores.
//
// Work unit: an "octet" of 8 rows (beam, token): 8 beams for T = 1, 4 beams x
// 2 tokens for T = 2 (row r = token r / 4, beam r % 4), one row per thread
// quad g.  A step-1 row takes k_0, d_0 and the decay of its beam's step-0 row
// from the partner lane (lane ^ 16), so both token counts run the same code and
// the same shared-memory footprint (two CTAs per SM).
//
// Data movement: each warp owns a run of octets and stages an octet's
// projection slices (the q, k, v, z head slices and the two gate words of each
// row) in shared memory with 16-byte cp.async copies, one octet ahead of the
// octet it computes.  S0 is staged once per CTA as an MN-major core-matrix
// image (the B operand).  The output tile goes back through the staged q slice
// and leaves as 16-byte stores.
//
// Contraction (tcgen05, A from tensor memory): the CTA's four warps work in
// rounds of one octet each.  Warp w writes its octet's normalised q rows to
// TMEM lanes 32w + g and k rows to lanes 32w + 8 + g (16x256b stores, bf16 hi
// and lo parts in two column ranges: ~16 mantissa bits of the fp32 q and k),
// one thread issues D/16 hi + D/16 lo MMAs of M = 128, N = D against S0 and
// commits to an mbarrier, and each warp reads its 16 accumulator lanes back
// with 16x256b loads, whose register layout is the m16n8 accumulator fragment
// (thread (g, tq): columns 8j + 2tq + {0, 1} of lanes g and g + 8).  The
// contraction order is free: a thread's pairs of channels 32m + 8tq + 2p + {0,1}
// go to TMEM column 8i + 2tq + e (i = 2m + p / 2, e = p % 2), i.e. MMA k index
// kappa = 32m + 16(p / 2) + 4tq + 2(p % 2) + {0,1}, and S0 row 32m + 8tq + 2p + d
// is staged as B row kappa (a bit permutation of the row index).
// TMEM per CTA: D accumulator columns, D/2 hi columns, D/2 lo columns.  The
// mbarrier wait is bounded and reports through the status word.
#include "gdn_mixer.cuh"
#include "tcgen05.cuh"

namespace kb {
namespace {

// warps per CTA: 8 for the first decode step (each warp fills 16 of its lane quadrant's 32
// TMEM lanes, so two warps share a quadrant and one M = 128 MMA serves both), 4 otherwise
template <int TMAX, bool CONT>
constexpr int mix_warps() { return TMAX == 1 && !CONT ? 8 : 4; }

template <int D>
struct MixLayout {
  static constexpr int CH = D / 8;          // 16-byte chunks in a head row
  static constexpr int NCH = 3 * D;         // conv channels: q head, k head, v head
  static constexpr int ROWB = 8 * D + 16;   // staged bytes per (token, beam): q, k, v, z, gate words
  static constexpr int S0B = D * D * 2;     // bf16 state, MN-major core-matrix image
  static constexpr int KGRP = 16 * D;       // bytes per group of 8 B rows (D / 8 core matrices)
  static constexpr int TCOLS = 2 * D;       // TMEM columns: accumulator, A hi, A lo
  static constexpr int TABB = 8 * NCH * 4;  // conv table [8][NCH] fp32
  static constexpr int NWB = D * 4;         // norm weight fp32
  static constexpr int OCTB = 8 * ROWB;     // one staged octet: 8 (beam, token) rows
  // continuation from a saved first step: a row also stages the parent token's raw q | k | v
  // slices and its gate word a
  static constexpr int ROWB_C = ROWB + 6 * D + 16;
  static constexpr int OCTB_C = 8 * ROWB_C;
  // shared memory of a CTA of `warps` warps, one staging buffer each (+ mbarrier, TMEM slot):
  // two CTAs per SM in every mode
  static constexpr size_t smem(bool cont, int warps) {
    return size_t(S0B) + TABB + NWB + size_t(warps) * (cont ? OCTB_C : OCTB) + 16;
  }
  static constexpr int REC = 4 * D;         // saved record per (beam, head): the token's delta, fp32
};

// MMA k index (B row) of state row r = 32m + 8tq + 2p + d: 32m + 16(p / 2) + 4tq + 2(p % 2) + d.
__device__ __forceinline__ int kappa_of(int r) {
  return (r & ~31) | (((r >> 2) & 1) << 4) | (((r >> 3) & 3) << 2) | (((r >> 1) & 1) << 1) | (r & 1);
}

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
// step t in {0, 1}, rounded to bf16 pairs:
//     conv_t = c_t + w3 x_t + [t = 1] w2 x_0
// (conv table rows 0..2: prefix-tap partial sums c_t, rows 3..6: taps w0..w3).
// `xt` / `x0` point at the raw bf16 inputs of steps t and 0 (equal when t = 0).
template <int NCH>
__device__ __forceinline__ void conv8_silu(const float* tab, int lc, int t, const unsigned char* xt,
                                           const unsigned char* x0, uint32_t out[4]) {
  const float4 c0 = *reinterpret_cast<const float4*>(tab + t * NCH + lc);
  const float4 c1 = *reinterpret_cast<const float4*>(tab + t * NCH + lc + 4);
  const float4 w30 = *reinterpret_cast<const float4*>(tab + 6 * NCH + lc);
  const float4 w31 = *reinterpret_cast<const float4*>(tab + 6 * NCH + lc + 4);
  const uint4 x = *reinterpret_cast<const uint4*>(xt);
  float2 acc[4];
  acc[0] = fma2(lo2(w30), bf2f(x.x), lo2(c0));
  acc[1] = fma2(hi2(w30), bf2f(x.y), hi2(c0));
  acc[2] = fma2(lo2(w31), bf2f(x.z), lo2(c1));
  acc[3] = fma2(hi2(w31), bf2f(x.w), hi2(c1));
  if (t) {  // lanes of step-1 rows; the step-0 lanes of the warp skip it
    const float4 w20 = *reinterpret_cast<const float4*>(tab + 5 * NCH + lc);
    const float4 w21 = *reinterpret_cast<const float4*>(tab + 5 * NCH + lc + 4);
    const uint4 y = *reinterpret_cast<const uint4*>(x0);
    acc[0] = fma2(lo2(w20), bf2f(y.x), acc[0]);
    acc[1] = fma2(hi2(w20), bf2f(y.y), acc[1]);
    acc[2] = fma2(lo2(w21), bf2f(y.z), acc[2]);
    acc[3] = fma2(hi2(w21), bf2f(y.w), acc[3]);
  }
#pragma unroll
  for (int p = 0; p < 4; ++p) out[p] = bf2_pack_f2(silu2(acc[p]));
}

// Same for one channel pair (lc even), returned as the exact bf16 values.
template <int NCH>
__device__ __forceinline__ float2 conv2_silu(const float* tab, int lc, int t, const unsigned char* xt,
                                             const unsigned char* x0) {
  float2 acc = fma2(*reinterpret_cast<const float2*>(tab + 6 * NCH + lc), bf2f(*reinterpret_cast<const uint32_t*>(xt)),
                    *reinterpret_cast<const float2*>(tab + t * NCH + lc));
  if (t) acc = fma2(*reinterpret_cast<const float2*>(tab + 5 * NCH + lc), bf2f(*reinterpret_cast<const uint32_t*>(x0)), acc);
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

// CONT (TMAX = 1): the second decode step from the first step's saved records -- octets
// of 8 beams, each row the beam's new token.  The parent token's delta comes from its
// record; its raw q | k | v (the conv window) and gate word a are staged, and its k,
// 1/|k| and decay are recomputed from them exactly as its own first step did.
template <int D, int TMAX, bool CONT, int NW = mix_warps<TMAX, CONT>()>
__global__ void __launch_bounds__(NW * 32, NW == 8 ? 2 : 1) gdn_mixer_kernel(const MixerArgs a, int octets_per_warp) {
  using L = MixLayout<D>;
  static_assert(!CONT || TMAX == 1, "the saved-state continuation stages one row per beam");
  constexpr int CH = L::CH, NCH = L::NCH, ROWB = CONT ? L::ROWB_C : L::ROWB, OCTB = CONT ? L::OCTB_C : L::OCTB;
  constexpr int NT = D / 8;      // n8 tiles of the V columns
  constexpr int NH = NT / 2;     // n8 tiles per half (bounds the accumulator registers)
  constexpr int KM = D / 32;     // 16-byte chunks per thread per head row
  constexpr int NI = D / 16;     // 8-column TMEM blocks of one A part (= MMA k16 steps)
  constexpr int BPO = 8 / TMAX;  // beams per octet; staged row r = (token r / BPO, beam r % BPO)
  constexpr long long kWait = 1ll << 31;
  constexpr uint32_t kIdesc = tc::idesc_bf16(128, D, 0, 1);  // A (TMEM) x MN-major S0
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* sS0 = smem;
  float* sTab = reinterpret_cast<float*>(smem + L::S0B);
  float* sNw = sTab + 8 * NCH;
  unsigned char* sStage = smem + L::S0B + L::TABB + L::NWB;
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sStage + NW * OCTB);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mbar + 1);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int tg = g / BPO;  // this thread's row: suffix step tg of beam g % BPO
  const int HV = a.HV;
  const int b = blockIdx.x / HV, hv = blockIdx.x % HV;
  const int h = hv / (HV / a.H);
  const int key_dim = a.H * D;
  const int conv_dim = 2 * key_dim + HV * D;
  const int64_t ld = a.ld_proj;
  const int octets = (a.W + BPO - 1) / BPO;
  const int oct0 = (blockIdx.y * NW + warp) * octets_per_warp;
  const int noct = max(0, min(octets_per_warp, octets - oct0));
  unsigned char* wbuf = sStage + warp * OCTB;
  // projection columns of the staged slices: q, k, v, z head slices; b and a gate words (aligned down)
  const int col_q = h * D, col_k = key_dim + h * D, col_v = 2 * key_dim + hv * D, col_z = conv_dim + hv * D;
  const int col_b = conv_dim + HV * D + hv, col_a = conv_dim + HV * D + HV + hv;

  // Projection row of (token tr, beam): rows (beam, t) of proj, or in continuation mode
  // the parent's row of the previous step (tr = 0) / the beam's row of the new token.
  auto parent_of = [&](int beam) { return min(max(a.parent[int64_t(b) * a.W + beam], 0), a.Wp - 1); };
  auto prow_of = [&](int tr, int beam) -> const __nv_bfloat16* {
    if (TMAX == 2 && a.proj_prev != nullptr) {
      if (tr == 0) {
        const int p = min(max(a.parent[int64_t(b) * a.W + beam], 0), a.Wp - 1);
        return a.proj_prev + (int64_t(b) * a.Wp + p) * ld;
      }
      return a.proj + (int64_t(b) * a.W + beam) * ld;
    }
    return a.proj + ((int64_t(b) * a.W + beam) * TMAX + tr) * ld;
  };
  // A warp stages an octet in two parts into its single buffer (the caller commits each as
  // a cp.async group): part qk (the rows' q | k slices and gate words; CONT: also the
  // parents' q | k slices and gate word a), read by the conv and the dot products, and part
  // vz (the rows' v | z slices; CONT: the parents' v slices), read by the recurrence and the
  // norm.  The next octet's part qk loads once this octet's conv is done and its part vz once
  // this octet's output has left, each behind the other half of the round; the output goes
  // out through the v slices (free after the recurrence).  Lane r & 7 resolves row r's
  // projection row once; the copies take it by shuffle (every lane's idx of one iteration
  // lies in the same row).
  auto stage_part = [&](int oct, unsigned char* buf, bool qk) {
    const int rl = lane & 7, beam_l = oct * BPO + rl % BPO;
    const bool ok_l = beam_l < a.W;
    const long long prow_l = reinterpret_cast<long long>(prow_of(rl / BPO, ok_l ? beam_l : 0));
#pragma unroll 4
    for (int idx = lane; idx < 8 * 2 * CH; idx += 32) {  // two slices of each row
      const int r = idx / (2 * CH), piece = (qk ? 0 : 2) + ((idx / CH) & 1), c = idx % CH;
      const __nv_bfloat16* prow = reinterpret_cast<const __nv_bfloat16*>(__shfl_sync(0xffffffffu, prow_l, r));
      const int col = piece < 2 ? (piece == 0 ? col_q : col_k) : (piece == 2 ? col_v : col_z);
      cp16z(buf + r * ROWB + piece * 2 * D + c * 16, prow + col + c * 8, oct * BPO + r % BPO < a.W);
    }
    if (qk) {  // lanes 0-15: the rows' gate words b, a
      const __nv_bfloat16* prow =
          reinterpret_cast<const __nv_bfloat16*>(__shfl_sync(0xffffffffu, prow_l, (lane >> 1) & 7));
      if (lane < 16) {
        const int r = lane >> 1, which = lane & 1;
        cp4z(buf + r * ROWB + 8 * D + which * 4, prow + ((which ? col_a : col_b) & ~1), oct * BPO + r % BPO < a.W);
      }
    }
    if constexpr (CONT) {
      const long long pp_l =
          reinterpret_cast<long long>(a.proj_prev + (int64_t(b) * a.Wp + parent_of(ok_l ? beam_l : 0)) * ld);
      const int per = qk ? 2 * CH : CH;  // the parents' q | k slices, or their v slices
#pragma unroll 4
      for (int idx = lane; idx < 8 * per; idx += 32) {
        const int r = idx / per, piece = qk ? (idx / CH) & 1 : 2, c = idx % CH;
        const __nv_bfloat16* pp = reinterpret_cast<const __nv_bfloat16*>(__shfl_sync(0xffffffffu, pp_l, r));
        cp16z(buf + r * ROWB + 8 * D + 16 + piece * 2 * D + c * 16,
              pp + (piece == 0 ? col_q : (piece == 1 ? col_k : col_v)) + c * 8, oct * BPO + r < a.W);
      }
      if (qk) {  // lanes 16-23: the parents' gate word a
        const __nv_bfloat16* pp = reinterpret_cast<const __nv_bfloat16*>(__shfl_sync(0xffffffffu, pp_l, lane & 7));
        if (lane >= 16 && lane < 24)
          cp4z(buf + (lane - 16) * ROWB + 14 * D + 16, pp + (col_a & ~1), oct * BPO + (lane - 16) < a.W);
      }
    }
  };

  // ---- CTA prologue: TMEM, S0 (B operand), this warp's first octet, conv table, norm weight ----
  if (warp == 0) tc::tmem_alloc(tslot, L::TCOLS);
  if (tid == 0) {
    tc::mbar_init(mbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  {
    const __nv_bfloat16* s0 = a.state + (int64_t(b) * HV + hv) * D * D;
    for (int idx = tid; idx < D * CH; idx += blockDim.x) {
      const int r = idx / CH, c = idx % CH, kap = kappa_of(r);
      cp_async16(sS0 + (kap >> 3) * L::KGRP + c * 128 + (kap & 7) * 16, s0 + r * D + c * 8);
    }
    cp_async_commit();
  }
  if (noct > 0) stage_part(oct0, wbuf, true);  // both parts of this warp's first octet
  cp_async_commit();
  if (noct > 0) stage_part(oct0, wbuf, false);
  cp_async_commit();
  // conv table: every thread's taps and prefix-state values are loaded before any is used
  constexpr int kTabIt = (NCH + NW * 32 - 1) / (NW * 32);
  float tw[kTabIt][4], ts[kTabIt][3];
#pragma unroll
  for (int i = 0; i < kTabIt; ++i) {
    const int c = tid + i * NW * 32;
    if (c < NCH) {
      int ch;
      if (c < D) ch = h * D + c;
      else if (c < 2 * D) ch = key_dim + h * D + (c - D);
      else ch = 2 * key_dim + hv * D + (c - 2 * D);
      const __nv_bfloat16* w = a.conv_weight + int64_t(ch) * 4;
      const __nv_bfloat16* s = a.conv_state + (int64_t(b) * conv_dim + ch) * a.conv_hist + a.conv_hist - 3;
#pragma unroll
      for (int e = 0; e < 4; ++e) tw[i][e] = __bfloat162float(w[e]);
#pragma unroll
      for (int e = 0; e < 3; ++e) ts[i][e] = __bfloat162float(s[e]);
    }
  }
  const float nwv = tid < D ? a.norm_weight[tid] : 0.f;
  const float neg_a = -expf(a.a_log[hv]), dtb = a.dt_bias[hv];
#pragma unroll
  for (int i = 0; i < kTabIt; ++i) {
    const int c = tid + i * NW * 32;
    if (c < NCH) {
      const float w0 = tw[i][0], w1 = tw[i][1], w2 = tw[i][2], w3 = tw[i][3];
      const float s0 = ts[i][0], s1 = ts[i][1], s2 = ts[i][2];
      sTab[0 * NCH + c] = w0 * s0 + w1 * s1 + w2 * s2;
      sTab[1 * NCH + c] = w0 * s1 + w1 * s2;
      sTab[2 * NCH + c] = w0 * s2;
      sTab[3 * NCH + c] = w0;  // tap applied to x_{t-3}
      sTab[4 * NCH + c] = w1;
      sTab[5 * NCH + c] = w2;
      sTab[6 * NCH + c] = w3;  // tap applied to x_t
      sTab[7 * NCH + c] = 0.f;
    }
  }
  static_assert(D <= NW * 32, "one norm weight per thread");
  if (tid < D) sNw[tid] = nwv;
  cp_async_wait<2>();       // S0 landed (the octet copies may still be in flight)
  tc::fence_async_smem();   // ... and visible to the tensor cores
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tslot;
  // this warp's 16 lanes (the first or second half of its lane quadrant): q rows g, k rows 8 + g
  const int lane0 = 32 * (warp & 3) + 16 * (warp >> 2);
  const uint32_t t_acc = tc::taddr(tmem, lane0, 0);
  const uint32_t t_hi = tc::taddr(tmem, lane0, D), t_lo = tc::taddr(tmem, lane0, D + D / 2);
  bool ok = true;

  // Rounds: every warp takes part in each round's barrier; a warp past its last octet
  // writes no A rows and reads nothing back (its TMEM lanes hold stale values).
  for (int it = 0; it < octets_per_warp; ++it) {
    const bool active = it < noct;
    unsigned char* buf = wbuf;
    // CONT: the parent's delta straight from its record into registers
    float2 d0s[CONT ? NT : 1];
    const int my_beam = (oct0 + it) * BPO + g % BPO;
    if constexpr (CONT) {
      const unsigned char* rec =
          a.saved + ((int64_t(b) * a.Wp + parent_of(active && my_beam < a.W ? my_beam : 0)) * HV + hv) * L::REC;
#pragma unroll
      for (int jj = 0; jj < NT; ++jj) d0s[jj] = *reinterpret_cast<const float2*>(rec + (jj * 8 + 2 * tq) * 4);
    }
    cp_async_wait<1>();  // this octet's part qk (its part vz may still be in flight)
    __syncwarp();

    unsigned char* rowg = buf + g * ROWB;  // this thread's row
    // the conv window's previous token: the same beam's step 0 (T = 2), or the parent's staged row
    const unsigned char* row0 = CONT ? rowg + 8 * D + 16 : (tg ? rowg - BPO * ROWB : rowg);
    constexpr int tsec = CONT ? 1 : 0;  // CONT rows are suffix step 1
    const int tt = CONT ? tsec : tg;

    // ---- q, k of this row (conv + SiLU, bf16), norms, gates, dot products --------------
    uint32_t qw[KM][4], kw[KM][4];
    float2 sq = make_float2(0.f, 0.f), sk = make_float2(0.f, 0.f);
#pragma unroll
    for (int m = 0; m < KM; ++m) {
      const int c = 4 * m + tq;
      conv8_silu<NCH>(sTab, 8 * c, tt, rowg + c * 16, row0 + c * 16, qw[m]);
      conv8_silu<NCH>(sTab, D + 8 * c, tt, rowg + 2 * D + c * 16, row0 + 2 * D + c * 16, kw[m]);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const float2 qf = bf2f(qw[m][p]), kf = bf2f(kw[m][p]);
        sq = fma2(qf, qf, sq);
        sk = fma2(kf, kf, sk);
      }
    }
    const float iq = 1.0f / sqrtf(quad_sum(sq.x + sq.y) + 1e-6f);
    const float ik = 1.0f / sqrtf(quad_sum(sk.x + sk.y) + 1e-6f);
    const float qs = iq * a.scale;
    float bt, at;
    {
      const __nv_bfloat162 bw = *reinterpret_cast<const __nv_bfloat162*>(rowg + 8 * D);
      const __nv_bfloat162 aw = *reinterpret_cast<const __nv_bfloat162*>(rowg + 8 * D + 4);
      bt = bf16r(sigmoid_f(__bfloat162float((col_b & 1) ? bw.y : bw.x)));
      at = expf(neg_a * softplus_f(__bfloat162float((col_a & 1) ? aw.y : aw.x) + dtb));
    }
    const float kq_self = chunk_dot<KM>(kw, qw) * ik * qs;  // k_t . q_t (normalised, q scaled)
    float At = at, ckq = 0.f, ckk = 0.f;
    if constexpr (TMAX == 2) {
      // step-1 rows: k_0, its norm and decay come from the step-0 partner row (lane ^ 16)
      uint32_t kp[KM][4];
#pragma unroll
      for (int m = 0; m < KM; ++m)
#pragma unroll
        for (int p = 0; p < 4; ++p) kp[m][p] = __shfl_xor_sync(0xffffffffu, kw[m][p], 16);
      const float ikp = __shfl_xor_sync(0xffffffffu, ik, 16), atp = __shfl_xor_sync(0xffffffffu, at, 16);
      const float dq = chunk_dot<KM>(kp, qw) * ikp * qs;  // k_0 . q_1
      const float dk = chunk_dot<KM>(kp, kw) * ikp * ik;  // k_0 . k_1
      if (tg) {
        At = atp * at;
        ckq = at * dq;
        ckk = at * dk;
      }
    }
    if constexpr (CONT) {
      // the parent token's k, 1/|k| and decay, recomputed from its staged raw row exactly as
      // its own first step computed them (conv at suffix step 0, the same summation order)
      uint32_t kp[KM][4];
      float2 skp = make_float2(0.f, 0.f);
#pragma unroll
      for (int m = 0; m < KM; ++m) {
        const int c = 4 * m + tq;
        conv8_silu<NCH>(sTab, D + 8 * c, 0, row0 + 2 * D + c * 16, row0 + 2 * D + c * 16, kp[m]);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float2 kf = bf2f(kp[m][p]);
          skp = fma2(kf, kf, skp);
        }
      }
      const float ikp = 1.0f / sqrtf(quad_sum(skp.x + skp.y) + 1e-6f);
      const __nv_bfloat162 apw = *reinterpret_cast<const __nv_bfloat162*>(row0 + 6 * D);
      const float atp = expf(neg_a * softplus_f(__bfloat162float((col_a & 1) ? apw.y : apw.x) + dtb));
      const float dq = chunk_dot<KM>(kp, qw) * ikp * qs;  // k_0 . q_1
      const float dk = chunk_dot<KM>(kp, kw) * ikp * ik;  // k_0 . k_1
      At = atp * at;
      ckq = at * dq;
      ckk = at * dk;
    }
    __syncwarp();  // part qk read: the next octet's part qk
    if (it + 1 < noct) stage_part(oct0 + it + 1, buf, true);
    cp_async_commit();
    // first decode step with a record buffer: this row's delta for the next step
    unsigned char* srec = nullptr;
    if constexpr (TMAX == 1 && !CONT) {
      if (a.save != nullptr && active && my_beam < a.W) srec = a.save + ((int64_t(b) * a.W + my_beam) * HV + hv) * L::REC;
    }

    // ---- A = [q ; k] (bf16 hi, lo) into TMEM; one thread runs the MMAs against S0 ---------
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      uint32_t ar[4 * NI];
#pragma unroll
      for (int m = 0; m < KM; ++m)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int i = 2 * m + hh;  // TMEM column block of channel pairs 2hh, 2hh + 1 of chunk 4m + tq
          const float2 q0 = mul2(bf2f(qw[m][2 * hh]), make_float2(qs, qs));
          const float2 q1 = mul2(bf2f(qw[m][2 * hh + 1]), make_float2(qs, qs));
          const float2 k0 = mul2(bf2f(kw[m][2 * hh]), make_float2(ik, ik));
          const float2 k1 = mul2(bf2f(kw[m][2 * hh + 1]), make_float2(ik, ik));
          const uint32_t h0 = bf2_pack_f2(q0), h1 = bf2_pack_f2(q1), h2 = bf2_pack_f2(k0), h3 = bf2_pack_f2(k1);
          if (part == 0) {
            ar[4 * i + 0] = h0;
            ar[4 * i + 1] = h1;
            ar[4 * i + 2] = h2;
            ar[4 * i + 3] = h3;
          } else {
            const float2 neg1 = make_float2(-1.f, -1.f);
            ar[4 * i + 0] = bf2_pack_f2(fma2(bf2f(h0), neg1, q0));
            ar[4 * i + 1] = bf2_pack_f2(fma2(bf2f(h1), neg1, q1));
            ar[4 * i + 2] = bf2_pack_f2(fma2(bf2f(h2), neg1, k0));
            ar[4 * i + 3] = bf2_pack_f2(fma2(bf2f(h3), neg1, k1));
          }
        }
      if constexpr (NI == 8) {
        if (part == 0) tc::st16x256b_x8(t_hi, ar); else tc::st16x256b_x8(t_lo, ar);
      } else {
        if (part == 0) tc::st16x256b_x4(t_hi, ar); else tc::st16x256b_x4(t_lo, ar);
      }
    }
    tc::wait_st();
    tc::fence_before();
    __syncthreads();
    if (tid == 0) {
      tc::fence_after();
      const uint32_t sb = smem_u32(sS0);
#pragma unroll
      for (int part = 0; part < 2; ++part)
#pragma unroll
        for (int st = 0; st < NI; ++st)
          tc::mma_bf16_ta(tmem, tmem + D + part * (D / 2) + 8 * st, tc::smem_desc(sb + st * 2 * L::KGRP, L::KGRP, 128),
                          kIdesc, part > 0 || st > 0);
      tc::commit(mbar);
    }
    if (!active) continue;
    ok = tc::mbar_wait(mbar, uint32_t(it) & 1u, kWait) && ok;
    tc::fence_after();
    cp_async_wait<1>();  // this octet's part vz (the next octet's part qk may still be in flight)
    __syncwarp();

    // ---- recurrence and gated RMSNorm over the accumulator, in two column halves ---------
    uint32_t ob[NT];
    float ss = 0.f;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      float acc[NH][4];
      {
        uint32_t r[4 * NH];
        if constexpr (NH == 8) tc::ld16x256b_x8(t_acc + hf * 64, r); else tc::ld16x256b_x4(t_acc + hf * 32, r);
        tc::wait_ld();
#pragma unroll
        for (int j = 0; j < NH; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[j][e] = __uint_as_float(r[4 * j + e]);
      }
      // columns (jj*8 + 2tq, +1): acc[j][0..1] = S0^T q, acc[j][2..3] = S0^T k of this row
#pragma unroll
      for (int j = 0; j < NH; ++j) {
        const int jj = hf * NH + j, col0 = jj * 8 + 2 * tq;
        const float2 vx = conv2_silu<NCH>(sTab, 2 * D + col0, tt, rowg + 4 * D + col0 * 2, row0 + 4 * D + col0 * 2);
        float2 skt = mul2(make_float2(At, At), make_float2(acc[j][2], acc[j][3]));
        float2 o = mul2(make_float2(At, At), make_float2(acc[j][0], acc[j][1]));
        const float2 nb = make_float2(-bt, -bt);
        float2 d = mul2(make_float2(bt, bt), vx);
        d = fma2(nb, skt, d);  // beta (v - S^T k)
        if constexpr (TMAX == 2) {
          const float2 d0 = make_float2(__shfl_xor_sync(0xffffffffu, d.x, 16), __shfl_xor_sync(0xffffffffu, d.y, 16));
          if (tg) {
            skt = fma2(make_float2(ckk, ckk), d0, skt);
            o = fma2(make_float2(ckq, ckq), d0, o);
            d = fma2(nb, skt, mul2(make_float2(bt, bt), vx));
          }
        }
        if constexpr (CONT) {
          const float2 d0 = d0s[jj];
          skt = fma2(make_float2(ckk, ckk), d0, skt);
          o = fma2(make_float2(ckq, ckq), d0, o);
          d = fma2(nb, skt, mul2(make_float2(bt, bt), vx));
        }
        if (srec != nullptr) *reinterpret_cast<float2*>(srec + col0 * 4) = d;
        o = fma2(d, make_float2(kq_self, kq_self), o);
        ob[jj] = bf2_pack_f2(o);  // gated_delta returns v's dtype
        const float2 of = bf2f(ob[jj]);
        ss = fmaf(of.x, of.x, fmaf(of.y, of.y, ss));
      }
    }
    // gated RMSNorm, written over this row's staged v slice once every row of the octet has
    // read its v slices (a step-1 row reads its step-0 row's too)
    constexpr int kOut = 4 * D;
    __syncwarp();
    const float inv = 1.0f / sqrtf(quad_sum(ss) / float(D) + a.norm_eps);
#pragma unroll
    for (int jj = 0; jj < NT; ++jj) {
      const int col = jj * 8 + 2 * tq;
      const float2 of = bf2f(ob[jj]);
      const float2 z = bf2f(*reinterpret_cast<const uint32_t*>(rowg + 6 * D + col * 2));
      const float2 w = *reinterpret_cast<const float2*>(sNw + col);
      const float2 sz = silu2(z);
      const float2 n = bf2f(bf2_pack(of.x * inv, of.y * inv));  // bf16(o * inv), the pair in one conversion
      const float2 h = bf2f(bf2_pack(w.x * n.x, w.y * n.y));    // bf16(w * .)
      *reinterpret_cast<uint32_t*>(rowg + kOut + col * 2) = bf2_pack(h.x * sz.x, h.y * sz.y);
    }
    __syncwarp();
    // ---- the octet's output rows, 16 bytes per store ------------------------------------
    const bool cont = TMAX == 2 && a.proj_prev != nullptr;  // continuation: the new token's rows only
    for (int idx = lane; idx < 8 * CH; idx += 32) {
      const int r = idx / CH, c = idx % CH;
      const int beam = (oct0 + it) * BPO + r % BPO;
      if (beam < a.W && (!cont || r / BPO == 1)) {
        const int64_t orow = cont ? int64_t(b) * a.W + beam : (int64_t(b) * a.W + beam) * TMAX + r / BPO;
        *reinterpret_cast<uint4*>(a.out + orow * (int64_t(HV) * D) + hv * D + c * 8) =
            *reinterpret_cast<const uint4*>(buf + r * ROWB + kOut + c * 16);
      }
    }
    __syncwarp();
    if (it + 1 < noct) stage_part(oct0 + it + 1, buf, false);  // part vz read: the next octet's part vz
    cp_async_commit();
  }
  cp_async_wait<0>();
  if (!ok && lane == 0) atomicOr(a.status, 1u);  // the MMA completion wait timed out
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::tmem_free(tmem, L::TCOLS);
  }
}

template <int D, int TMAX, bool CONT = false>
int launch_mixer(const MixerArgs& a, cudaStream_t stream) {
  using L = MixLayout<D>;
  constexpr int NW = mix_warps<TMAX, CONT>();
  auto kern = gdn_mixer_kernel<D, TMAX, CONT, NW>;
  constexpr size_t smem = L::smem(CONT, NW);
  static_assert(2 * (smem + 1024) <= 233472, "two CTAs per SM");
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
    set_error("gdn mixer: cannot reserve %zu bytes of shared memory", smem);
    return KADLLM_ECUDA;
  }
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  constexpr int bpo = 8 / TMAX;
  const int octets = (a.W + bpo - 1) / bpo;
  // split a head's octets over enough CTAs for about two waves (two CTAs per SM), each
  // warp taking a run of consecutive octets
  const int heads = a.B * a.HV;
  int ny = (4 * sms + heads - 1) / heads;
  ny = max(1, min(ny, (octets + NW - 1) / NW));
  const int opw = (octets + NW * ny - 1) / (NW * ny);
  ny = (octets + NW * opw - 1) / (NW * opw);
  const dim3 grid{unsigned(heads), unsigned(ny)};
  kern<<<grid, NW * 32, smem, stream>>>(a, opw);
  KB_CHECK_LAUNCH("gdn mixer launch");
  return KADLLM_OK;
}

}  // namespace

bool gdn_mixer_staged_ok(const MixerArgs& a) {
  if (!(a.D == 64 || a.D == 128) || a.T < 1 || a.T > 2 || a.conv_hist < 3) return false;
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return a.status != nullptr && al16(a.proj) && al16(a.out) && al16(a.state) && a.ld_proj % 8 == 0 &&
         (a.proj_prev == nullptr || (a.T == 2 && al16(a.proj_prev))) && (a.save == nullptr || (a.T == 1 && al16(a.save))) &&
         (a.saved == nullptr || (a.T == 2 && a.proj_prev != nullptr && al16(a.saved)));
}

int gdn_mixer_staged(const MixerArgs& a, cudaStream_t stream) {
  if (a.saved != nullptr)  // the second step from the first step's records: one row per beam
    return a.D == 128 ? launch_mixer<128, 1, true>(a, stream) : launch_mixer<64, 1, true>(a, stream);
  if (a.D == 128) return a.T == 1 ? launch_mixer<128, 1>(a, stream) : launch_mixer<128, 2>(a, stream);
  return a.T == 1 ? launch_mixer<64, 1>(a, stream) : launch_mixer<64, 2>(a, stream);
}

int64_t gdn_mixer_record_bytes(int64_t rows, int64_t v_heads, int64_t dim) {
  return rows * v_heads * 4 * dim;
}

}  // namespace kb
