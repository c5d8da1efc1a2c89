// Prompt prefill of the Gated-DeltaNet layers in the WY form of the chunked
// gated delta rule: a parallel per-chunk preparation and a lean sequential
// state scan (BF16 activations and operands, fp32 accumulation and state).
//
// Semantics: Transformers Qwen3_5GatedDeltaNet.forward on the prompt
// (transformers/models/qwen3_5/modeling_qwen3_5.py:422-533): causal conv1d +
// SiLU (zero left padding), beta = sigmoid(b), g = -exp(A_log) softplus(a +
// dt_bias), q/k L2-normalised (fp32), torch_chunk_gated_delta_rule (chunk 64,
// modeling_qwen3_5.py:234-311) and the gated RMSNorm (modeling_qwen3_5.py:
// 175-190), plus the request-sized prefix the decode replays from: the last 4
// pre-conv columns and the final recurrent state, BF16 like the hybrid cache
// (transformers/cache_utils.py:734-800).  The WY quantities are the
// reference's own: value = T (v beta) and k_cumdecay = T (k beta e^g) with
// T = (I + L)^-1, L = strictly-lower(diag(beta) K K^T o exp(G_i - G_j)).
//
// prep (grid: chunks x B*HV, 8 warps, 2 CTAs per SM) -- everything that does
//       not depend on the recurrent state, for all chunks at once:
//         the head's q / k / v projection columns (+ 3-token halo) staged by
//         cp.async, conv + SiLU, q (scaled) / k L2 norm, gates, in-chunk
//         cumulative decay G, K K^T and Q K^T on the tensor cores, T by 16x16
//         forward substitution plus two levels of TF32 block merges
//         [[A,0],[C,D]]^-1 = [[A^-1,0],[-D^-1 C A^-1, D^-1]], then
//         W = T diag(beta e^G) K and U = T diag(beta) V on the tensor cores.
//       Writes one contiguous block per chunk: Q' = e^G q | K' = e^{G_last - G} k | W | U |
//       Aqk = (Q K^T o exp(G_i - G_j)) lower incl. diagonal | G.
// scan  (grid: B*HV, 8 warps) -- per chunk, with the next block prefetched by
//       cp.async, three barriers:
//         [W; Q'] S (one pass over S)      Vn = U - W S,  O = Q' S  (Q' = e^G q)
//         S <- e^{G_last} S + K'^T Vn      O += Aqk Vn -> gated RMSNorm -> out
//       (the tensor-core scan normalises chunk c's output rows while chunk c + 1's
//       first MMA runs)
// S stays in fp32 MMA accumulators, with a BF16 copy in shared memory as the B
// operand of the next chunk.
#include "mma_tiles.cuh"
#include "tcgen05.cuh"

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
  unsigned char* blocks;                       // [B*HV, nc] chunk blocks (ChunkBlock)
  uint32_t* status;                            // bit 0: a tensor-core wait of the scan timed out
  int tc_layout;                               // chunk blocks in the tensor-core scan's shared-memory image
  const int* cu;                               // varlen: request b = rows [cu[b], cu[b+1]) (null: b*L .. +L)
  int64_t rows;                                // rows of proj / out (B*L, or cu[B])
  int B, L, nc, H, HV;                         // L, nc: the (longest) request's length and chunk count
  float scale;
};

// One chunk's prep output in the workspace.  Dense rows, or (tc_layout, DK = DV =
// 128) the tensor-core scan's shared-memory image: w, q, kp as one 128-row
// K-major core-matrix tile [W; Q'] followed by K' (the same byte order read as
// MN-major), Aqk as a 64-wide K-major core tile, U as 256-byte rows with XOR-
// swizzled 16-byte chunks; so the scan stages a chunk with one bulk copy.
template <int DK, int DV>
struct ChunkBlock {
  static constexpr size_t w = 0;                           // [kC][DK] bf16, T diag(beta e^G) K
  static constexpr size_t q = w + size_t(kC) * DK * 2;     // [kC][DK] bf16, e^{G_i} q_i (normalised, scaled)
  static constexpr size_t kp = q + size_t(kC) * DK * 2;    // [kC][DK] bf16, e^{G_last - G_i} k_i
  static constexpr size_t aqk = kp + size_t(kC) * DK * 2;  // [kC][kC] bf16
  static constexpr size_t u = aqk + size_t(kC) * kC * 2;   // [kC][DV] bf16, T diag(beta) V
  static constexpr size_t g = u + size_t(kC) * DV * 2;     // [kC] f32, cumulative log decay
  static constexpr size_t bytes = g + size_t(kC) * 4;
  static_assert(bytes % 16 == 0, "16-byte blocks");
};

// 16-byte unit o of a block region in the tensor-core image -> (row, 16-byte chunk) of the source tile.
__device__ __forceinline__ void core16_rc(int o, int& r, int& ch) { r = ((o >> 7) << 3) | (o & 7); ch = (o >> 3) & 15; }
__device__ __forceinline__ void core8_rc(int o, int& r, int& ch) { r = ((o >> 6) << 3) | (o & 7); ch = (o >> 3) & 7; }
__device__ __forceinline__ void swz16_rc(int o, int& r, int& ch) { r = o >> 4; ch = (o & 15) ^ (r & 7); }

// Request b's first row and length (packed varlen rows, or B requests of L rows).
__device__ __forceinline__ void seq_of(const SplitArgs& a, int b, int64_t& row0, int& len) {
  if (a.cu) {
    row0 = a.cu[b];
    len = a.cu[b + 1] - a.cu[b];
  } else {
    row0 = int64_t(b) * a.L;
    len = a.L;
  }
}

// Named barrier `id` over the first n threads of the CTA.
__device__ __forceinline__ void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(n) : "memory"); }

template <int DK, int DV>
size_t workspace_bytes(int64_t B, int64_t HV, int64_t L) {
  const int64_t nc = (L + kC - 1) / kC;
  return size_t(B * HV * nc) * ChunkBlock<DK, DV>::bytes + 256;
}

// ---------------------------------------------------------------------------
// prep
// ---------------------------------------------------------------------------
template <int DK, int DV>
struct PrepSmem {
  static constexpr int NCH = 2 * DK + DV;            // q | k | v channels of the head
  static constexpr int RS = NCH + 8, SQ = DK + 8, SV = DV + 8, SL = kC + 1, ST = kC + 8;
  // region R: raw projection tile [kC + 3][RS] (rows = tokens t0-3 .. t0+63), then
  // after the conv: L (fp32) | tmp | T1 | T2 | Aqk (bf16)
  static constexpr size_t l = 0;
  static constexpr size_t tmp = l + size_t(kC) * SL * 4;
  static constexpr size_t t1 = tmp + size_t(32) * 33 * 4;
  static constexpr size_t t2 = t1 + size_t(kC) * ST * 2;
  static constexpr size_t a = t2 + size_t(kC) * ST * 2;
  static constexpr size_t r_end = a + size_t(kC) * ST * 2;
  static constexpr size_t raw_bytes = size_t(kC + 3) * RS * 2;
  static constexpr size_t r_bytes = ((raw_bytes > r_end ? raw_bytes : r_end) + 15) / 16 * 16;
  static constexpr size_t q = r_bytes;                       // q, later W
  static constexpr size_t k = q + size_t(kC) * SQ * 2;       // k, later K'
  static constexpr size_t v = k + size_t(kC) * SQ * 2;       // v, later U
  static constexpr size_t vec = v + size_t(kC) * SV * 2;     // G | beta | raw g | e^G | beta e^G | e^{G_last - G}
  static constexpr size_t cw = vec + size_t(kC) * 4 * 6;     // the head's conv taps [NCH][4] bf16
  static constexpr size_t bytes = cw + size_t(NCH) * 4 * 2;
  static_assert(t1 % 16 == 0 && a % 16 == 0 && q % 16 == 0 && k % 16 == 0 && v % 16 == 0 && cw % 16 == 0, "alignment");
};

// Copy a [kC][COLS] bf16 tile from padded shared rows to global, 16 bytes a thread, consecutive
// threads on consecutive destination bytes: dense rows (kind 0) or a tensor-core image (kind 1
// core16, 2 core8, 3 swizzled rows).  scale (per row) multiplies the values when given.
template <int COLS>
__device__ __forceinline__ void export_tile(unsigned char* dst, const __nv_bfloat16* src, int lds, int kind,
                                            const float* scale, int tid, int nthreads) {
  constexpr int CH = COLS / 8;
  for (int o = tid; o < kC * CH; o += nthreads) {
    int r, ch;
    if (kind == 1) core16_rc(o, r, ch);
    else if (kind == 2) core8_rc(o, r, ch);
    else if (kind == 3) swz16_rc(o, r, ch);
    else { r = o / CH; ch = o % CH; }
    uint4 raw = *reinterpret_cast<const uint4*>(src + r * lds + ch * 8);
    if (scale) {
      const float f = scale[r];
      __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) hh[j] = __floats2bfloat162_rn(__low2float(hh[j]) * f, __high2float(hh[j]) * f);
    }
    reinterpret_cast<uint4*>(dst)[o] = raw;
  }
}

template <int DK, int DV>
__global__ void __launch_bounds__(256, 2) gdn_prep_kernel(const SplitArgs a) {
  using M = PrepSmem<DK, DV>;
  using CB = ChunkBlock<DK, DV>;
  constexpr int NCH = M::NCH, RS = M::RS, SQ = M::SQ, SV = M::SV, SL = M::SL, ST = M::ST;
  constexpr int NT = 256;
  extern __shared__ __align__(16) unsigned char smem[];
  __nv_bfloat16* sRawT = reinterpret_cast<__nv_bfloat16*>(smem);  // [kC + 3][RS]
  float* sL = reinterpret_cast<float*>(smem + M::l);
  float* sTmp = reinterpret_cast<float*>(smem + M::tmp);          // [32][33]
  __nv_bfloat16* sT1 = reinterpret_cast<__nv_bfloat16*>(smem + M::t1);
  __nv_bfloat16* sT2 = reinterpret_cast<__nv_bfloat16*>(smem + M::t2);
  __nv_bfloat16* sA = reinterpret_cast<__nv_bfloat16*>(smem + M::a);
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem + M::q);
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smem + M::k);
  __nv_bfloat16* sV = reinterpret_cast<__nv_bfloat16*>(smem + M::v);
  float* sG = reinterpret_cast<float*>(smem + M::vec);
  float* sBeta = sG + kC;
  float* sRaw = sBeta + kC;
  float* sEG = sRaw + kC;     // e^{G_i}
  float* sBEG = sEG + kC;     // beta_i e^{G_i}
  float* sEGL = sBEG + kC;    // e^{G_last - G_i}
  __nv_bfloat16* sCw = reinterpret_cast<__nv_bfloat16*>(smem + M::cw);  // [NCH][4] conv taps of the head

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = blockIdx.x;
  const int bh = blockIdx.y, b = bh / a.HV, hv = bh % a.HV, h = hv / (a.HV / a.H);
  const int key_dim = a.H * DK, conv_dim = 2 * key_dim + a.HV * DV;
  const int t0 = c * kC;
  auto chan = [&](int lc) {  // head-local channel -> projection column
    return lc < DK ? h * DK + lc : (lc < 2 * DK ? key_dim + h * DK + (lc - DK) : 2 * key_dim + hv * DV + (lc - 2 * DK));
  };
  int64_t seq0;
  int L;
  seq_of(a, b, seq0, L);
  if (t0 >= L) return;  // past this request's last chunk (varlen): the whole CTA, before any barrier
  const __nv_bfloat16* prow0 = a.proj + seq0 * a.ld_proj;

  // ---- stage the raw projection tile (tokens t0-3 .. t0+63, zero outside [0, L)) -----
  {  // each thread keeps one 16-byte column chunk and walks the rows GRP at a time
    constexpr int CPR = NCH / 8, GRP = NT / CPR;  // chunks per staged row, rows staged at once
    static_assert(GRP >= 1, "a block stages at least one row at a time");
    if (tid < GRP * CPR) {
      const int lc = (tid % CPR) * 8;
      const __nv_bfloat16* src = prow0 + chan(lc);
      __nv_bfloat16* dst = sRawT + lc;
      for (int r = tid / CPR; r < kC + 3; r += GRP) {
        const int t = t0 - 3 + r;
        if (t >= 0 && t < L) cp_async16(dst + r * RS, src + int64_t(t) * a.ld_proj);
        else *reinterpret_cast<uint4*>(dst + r * RS) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    for (int i = tid; i < NCH / 2; i += NT)  // conv taps: 16 bytes = two channels' four taps
      cp_async16(sCw + i * 8, a.conv_w + int64_t(chan(2 * i)) * 4);
  }
  cp_async_commit();
  float gb = 0.f, ga = 0.f;  // gate inputs of token t0 + tid
  if (tid < kC && t0 + tid < L) {
    const __nv_bfloat16* pr = prow0 + int64_t(t0 + tid) * a.ld_proj + conv_dim + int64_t(a.HV) * DV;
    gb = __bfloat162float(pr[hv]);
    ga = __bfloat162float(pr[a.HV + hv]);
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- conv + SiLU: 8 channels x 4 tokens per item, from the staged tile, in fp32 pairs -
  constexpr int NG = NCH / 8, SEG = 4;
  for (int item = tid; item < NG * (kC / SEG); item += NT) {
    const int grp = item % NG, seg = item / NG;
    const int lc = grp * 8;
    float2 w2[4][4];  // [channel pair][tap]
    {
      const uint4* wp = reinterpret_cast<const uint4*>(sCw + lc * 4);
#pragma unroll
      for (int u = 0; u < 4; ++u) {  // uint4 u = taps of channels 2u, 2u + 1
        const uint4 raw = wp[u];
        const float2 c0a = bf2f(raw.x), c0b = bf2f(raw.y), c1a = bf2f(raw.z), c1b = bf2f(raw.w);
        w2[u][0] = make_float2(c0a.x, c1a.x);
        w2[u][1] = make_float2(c0a.y, c1a.y);
        w2[u][2] = make_float2(c0b.x, c1b.x);
        w2[u][3] = make_float2(c0b.y, c1b.y);
      }
    }
    auto row4 = [&](int r, float2 (&v)[4]) {  // staged row r = token t0 - 3 + r, 8 channels as 4 pairs
      const uint4 u = *reinterpret_cast<const uint4*>(sRawT + r * RS + lc);
      v[0] = bf2f(u.x);
      v[1] = bf2f(u.y);
      v[2] = bf2f(u.z);
      v[3] = bf2f(u.w);
    };
    const int r0 = seg * SEG;
    float2 win[3][4];
    row4(r0, win[0]);
    row4(r0 + 1, win[1]);
    row4(r0 + 2, win[2]);
    __nv_bfloat16* dst = lc < DK ? sQ + lc : (lc < 2 * DK ? sK + (lc - DK) : sV + (lc - 2 * DK));
    const int ld = lc < 2 * DK ? SQ : SV;
#pragma unroll
    for (int r = r0; r < r0 + SEG; ++r) {
      float2 x[4];
      row4(r + 3, x);
      uint4 u = make_uint4(0u, 0u, 0u, 0u);
      if (t0 + r < L) {
        uint32_t* uw = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
        for (int pp = 0; pp < 4; ++pp) {
          float2 acc = mul2(win[0][pp], w2[pp][0]);
          acc = fma2(win[1][pp], w2[pp][1], acc);
          acc = fma2(win[2][pp], w2[pp][2], acc);
          acc = fma2(x[pp], w2[pp][3], acc);
          const float2 o = silu2(acc);
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(o.x, o.y);
          uw[pp] = *reinterpret_cast<const uint32_t*>(&h2);
        }
      }
      *reinterpret_cast<uint4*>(dst + r * ld) = u;
#pragma unroll
      for (int pp = 0; pp < 4; ++pp) {
        win[0][pp] = win[1][pp];
        win[1][pp] = win[2][pp];
        win[2][pp] = x[pp];
      }
    }
  }
  if (t0 + kC >= L) {  // last chunk: conv state = pre-conv columns of tokens L-4 .. L-1 (staged rows L-1-t0 ..)
    for (int lc = tid; lc < NCH; lc += NT) {
      __nv_bfloat16 s4[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) s4[j] = sRawT[(L - 1 - t0 + j) * RS + lc];
      *reinterpret_cast<uint2*>(a.conv_state + (int64_t(b) * conv_dim + chan(lc)) * 4) = *reinterpret_cast<uint2*>(s4);
    }
  }
  // ---- gates ------------------------------------------------------------------------
  if (tid < kC) {
    float g = 0.f, be = 0.f;
    if (t0 + tid < L) {
      be = bf16r(sigmoid_f(gb));
      g = -expf(a.a_log[hv]) * softplus_f(ga + a.dt_bias[hv]);
    }
    sRaw[tid] = g;
    sBeta[tid] = be;
  }
  __syncthreads();
  // ---- L2 normalisation of q (scaled) and k, in place ---------------------------------
  if (tid < 2 * kC) {
    const int r = tid & (kC - 1), part = tid >> 6;  // 64 rows x {q, k}
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
#pragma unroll
    for (int u = 0; u < DK / 8; ++u) {
      uint4 raw = *reinterpret_cast<const uint4*>(row + u * 8);
      __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) hh[j] = __floats2bfloat162_rn(__low2float(hh[j]) * f, __high2float(hh[j]) * f);
      *reinterpret_cast<uint4*>(row + u * 8) = raw;
    }
  } else if (warp == 4) {  // in-chunk cumulative log decay (warp scan over 64 values)
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
  }
  __syncthreads();
  if (tid < kC) {  // per-token decay factors (read after later barriers)
    const float e = __expf(sG[tid]);
    sEG[tid] = e;
    sBEG[tid] = sBeta[tid] * e;
    sEGL[tid] = __expf(sG[kC - 1] - sG[tid]);
  }
  // in-chunk decay matrix exp(G_i - G_j), lower triangle incl. the diagonal (zero above), once
  // per chunk for both epilogues below; it lives in the T1 / T2 area, written only later
  constexpr int SD = kC + 8;  // row stride: 8-byte aligned pairs, conflict-free half-warp reads
  float* sDec = reinterpret_cast<float*>(smem + M::t1);  // [kC][SD]
  static_assert(M::t1 + size_t(kC) * SD * 4 <= M::a, "decay matrix fits the T1 / T2 area");
  for (int e = tid; e < kC * kC; e += NT) {
    const int i = e / kC, j = e % kC;
    sDec[i * SD + j] = i >= j ? __expf(sG[i] - sG[j]) : 0.f;
  }
  const int g8 = lane >> 2, tq = lane & 3;
  // ---- warps 0-3: K K^T -> L (fp32); warps 4-7: Q K^T -> Aqk (bf16) --------------------
  {
    const int mt = warp & 3;
    const bool is_q = warp >= 4;
    float acc[8][4];
    zero_acc<8>(acc);
    warp_mma<DK, 8, false, false>(acc, is_q ? sQ : sK, SQ, mt * 16, 0, sK, SQ, 0, 0);
    __syncthreads();  // the decay matrix is complete
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int i = mt * 16 + g8 + hr * 8;
        const int col = j * 8 + tq * 2;
        const float2 dec2 = *reinterpret_cast<const float2*>(sDec + i * SD + col);
        float av[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int cc = col + e;
          const float dec = e ? dec2.y : dec2.x;
          if (is_q) av[e] = acc[j][hr * 2 + e] * dec;
          else sL[i * SL + cc] = i > cc ? sBeta[i] * acc[j][hr * 2 + e] * dec : 0.f;
        }
        if (is_q) *reinterpret_cast<__nv_bfloat162*>(sA + i * ST + col) = __floats2bfloat162_rn(av[0], av[1]);
      }
  }
  __syncthreads();
  // ---- T = (I + L)^-1 (warps 0-3; all threads meet every barrier) -----------------------
  if (tid < kC) {  // diagonal 16x16 blocks: lane (block, column j) forward-substitutes column j in registers
    const int d0 = (tid >> 4) * 16, j = tid & 15;
    const float* Lb = sL + d0 * SL + d0;
    float t[16];  // T[i][j] of this block; T = (I + L)^-1 is unit lower triangular
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int m = 0; m < i; ++m) acc = fmaf(Lb[i * SL + m], t[m], acc);  // t[m] = 0 for m < j
      t[i] = i < j ? 0.f : (i == j ? 1.f : -acc);
    }
    __syncwarp();  // a block's 16 lanes share a warp: every read of L precedes the writes
#pragma unroll
    for (int i = 1; i < 16; ++i)
      if (i > j) sL[(d0 + i) * SL + d0 + j] = t[i];
  }
  __syncthreads();
  if (tid < kC) sL[tid * SL + tid] = 1.f;  // sL now holds unit-lower blocks (zeros above)
  __syncthreads();
  {  // level 1 (16x16 blocks, TF32): T_10 = -T_11 (L_10 T_00), T_32 = -T_33 (L_32 T_22)
    const int bp = (warp & 3) >> 1, nc8 = warp & 1;  // warp -> (block pair, 8-column half)
    const int r0 = 16 + 32 * bp, c0 = 32 * bp;
    float acc[1][4];
    zero_acc<1>(acc);
    if (warp < 4) {
      warp_mma_tf32<16, 1>(acc, sL + r0 * SL + c0, SL, sL + c0 * SL + c0 + nc8 * 8, SL);
      store_acc<1>(sTmp + bp * 16 * 33 + nc8 * 8, 33, acc, 1.f);
    }
    __syncthreads();
    zero_acc<1>(acc);
    if (warp < 4) warp_mma_tf32<16, 1>(acc, sL + r0 * SL + r0, SL, sTmp + bp * 16 * 33 + nc8 * 8, 33);
    __syncthreads();
    if (warp < 4) store_acc<1>(sL + r0 * SL + c0 + nc8 * 8, SL, acc, -1.f);
  }
  __syncthreads();
  {  // level 2 (32x32 blocks): T_[2:4][0:2] = -T_D (C T_A) with C = L[32:64, 0:32]
    const int mt = (warp & 3) >> 1, nh = warp & 1;  // 2 m-tiles x 2 column halves of 16
    float acc[2][4];
    zero_acc<2>(acc);
    if (warp < 4) {
      warp_mma_tf32<32, 2>(acc, sL + (32 + mt * 16) * SL, SL, sL + nh * 16, SL);
      store_acc<2>(sTmp + mt * 16 * 33 + nh * 16, 33, acc, 1.f);
    }
    __syncthreads();
    zero_acc<2>(acc);
    if (warp < 4) warp_mma_tf32<32, 2>(acc, sL + (32 + mt * 16) * SL + 32, SL, sTmp + nh * 16, 33);
    __syncthreads();
    if (warp < 4) store_acc<2>(sL + (32 + mt * 16) * SL + nh * 16, SL, acc, -1.f);
  }
  __syncthreads();
  // ---- T1 = T diag(beta e^G), T2 = T diag(beta) (bf16); export q ----------------------
  unsigned char* blk = a.blocks + (int64_t(bh) * a.nc + c) * CB::bytes;
  for (int e = tid * 2; e < kC * kC; e += NT * 2) {
    const int i = e / kC, j = e % kC;
    const float v0 = i >= j ? sL[i * SL + j] : 0.f;
    const float v1 = i >= j + 1 ? sL[i * SL + j + 1] : 0.f;
    *reinterpret_cast<__nv_bfloat162*>(sT1 + i * ST + j) = __floats2bfloat162_rn(v0 * sBEG[j], v1 * sBEG[j + 1]);
    *reinterpret_cast<__nv_bfloat162*>(sT2 + i * ST + j) = __floats2bfloat162_rn(v0 * sBeta[j], v1 * sBeta[j + 1]);
  }
  const bool tcl = DK == 128 && DV == 128 && a.tc_layout;
  // Q' = e^{G_i} q_i (the decay of the inter-chunk term, folded into the operand)
  export_tile<DK>(blk + CB::q, sQ, SQ, tcl ? 1 : 0, sEG, tid, NT);
  __syncthreads();
  // ---- warps 0-3: W = T1 K; warps 4-7: U = T2 V (tensor cores) ------------------------
  {
    static_assert(DK == DV && SQ == SV, "W and U share one tile shape");
    float acc[DK / 8][4];
    zero_acc<DK / 8>(acc);
    const int mt = warp & 3;
    warp_mma<kC, DK / 8, false, true>(acc, warp < 4 ? sT1 : sT2, ST, mt * 16, 0, warp < 4 ? sK : sV, SQ, 0, 0);
    __syncthreads();  // all reads of sK / sV done: overwrite with W (into sQ), U (into sV), K' (in sK)
    __nv_bfloat16* dst = warp < 4 ? sQ : sV;
#pragma unroll
    for (int j = 0; j < DK / 8; ++j) {
      const int r = mt * 16 + g8, col = j * 8 + tq * 2;
      *reinterpret_cast<__nv_bfloat162*>(dst + r * SQ + col) = __floats2bfloat162_rn(acc[j][0], acc[j][1]);
      *reinterpret_cast<__nv_bfloat162*>(dst + (r + 8) * SQ + col) = __floats2bfloat162_rn(acc[j][2], acc[j][3]);
    }
    for (int e = tid; e < kC * (DK / 8); e += NT) {  // K' = e^{G_last - G_i} k_i, 16 bytes at a time
      const int i = e / (DK / 8), cc = (e % (DK / 8)) * 8;
      uint4* p = reinterpret_cast<uint4*>(sK + i * SQ + cc);
      const float f = sEGL[i];
      uint4 raw = *p;
      __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) hh[j] = __floats2bfloat162_rn(__low2float(hh[j]) * f, __high2float(hh[j]) * f);
      *p = raw;
    }
  }
  __syncthreads();
  export_tile<DK>(blk + CB::kp, sK, SQ, tcl ? 1 : 0, nullptr, tid, NT);
  export_tile<DK>(blk + CB::w, sQ, SQ, tcl ? 1 : 0, nullptr, tid, NT);
  export_tile<DV>(blk + CB::u, sV, SV, tcl ? 3 : 0, nullptr, tid, NT);
  export_tile<kC>(blk + CB::aqk, sA, ST, tcl ? 2 : 0, nullptr, tid, NT);
  if (tid < kC / 4) reinterpret_cast<float4*>(blk + CB::g)[tid] = reinterpret_cast<const float4*>(sG)[tid];
}

// ---------------------------------------------------------------------------
// prep on the 5th-generation tensor cores (DK = DV = 128, tensor-core block layout)
// ---------------------------------------------------------------------------
// The chunk's raw (un-normalised) bf16 conv outputs k, q, v sit in shared-memory
// images in the core-matrix layout [token/8][feature/8][token%8][16 bytes] with a
// 144-byte feature-chunk stride (16-byte writes spread over the banks).  Read with
// rows = tokens they are K-major operands (SBO 2304, LBO 144); read with K = tokens,
// N = features they are MN-major operands (SBO 144, LBO 2304).  k and q are adjacent,
// so [K; Q] is one 128-row operand:
//   MMA1  [K; Q] K^T (M 128, N 64, K 128): K K^T and Q K^T, scaled afterwards by the
//         inverse L2 norms (the products of the bf16 conv outputs are exact in fp32)
//   MMA2  [T1; T2] K and [T1; T2] V (M 128, N 128, K 64): W = T1 K (rows 0-63 of the
//         first), U = T2 V (rows 64-127 of the second), with T1 = T diag(beta e^G / |k|),
//         T2 = T diag(beta).
// Epilogues run a thread per TMEM lane (row) and write the chunk block straight to
// global memory in the tensor-core scan's image order (coalesced 16-byte stores);
// Q' and K' are scaled copies of the q / k images, exported by warps 4-7 while
// warps 0-3 invert (I + L).
struct PrepTc {
  static constexpr int D = 128, NCH = 3 * D, RS = NCH + 8, SL = kC + 1;
  static constexpr int CST = 144;       // feature-chunk stride of an image
  static constexpr int GST = 16 * CST;  // 8-token group stride
  static constexpr int IMG = 8 * GST;   // one 64-token image
  static constexpr size_t raw_bytes = size_t(kC + 3) * RS * 2;  // staged projection tile (conv input)
  // after the conv the raw region holds L / T (fp32), the merge scratch and [T1; T2]
  static constexpr size_t l = 0;
  static constexpr size_t tmp = l + size_t(kC) * SL * 4;
  static constexpr size_t t12 = (tmp + size_t(32) * 33 * 4 + 127) / 128 * 128;  // K-major, SBO 1024, LBO 128
  static constexpr size_t k = (raw_bytes + 127) / 128 * 128;  // images k | q | v
  static constexpr size_t q = k + IMG;
  static constexpr size_t v = q + IMG;
  static constexpr size_t vec = v + IMG;  // 11 x [kC] fp32
  static constexpr size_t cw = vec + size_t(11) * kC * 4;
  static constexpr size_t bar = cw + size_t(NCH) * 4 * 2;
  static constexpr size_t slot = bar + 8;
  static constexpr size_t bytes = slot + 8;
  static_assert(t12 + size_t(2 * kC) * kC * 2 <= raw_bytes, "[T1; T2] fits the raw region");
  static_assert(bytes <= 115 * 1024, "two CTAs per SM");
  __device__ static uint32_t img_off(int t, int ch) { return (t >> 3) * GST + ch * CST + (t & 7) * 16; }
};

__global__ void __launch_bounds__(256, 2) gdn_prep_tc_kernel(const SplitArgs a) {
  using M = PrepTc;
  using CB = ChunkBlock<128, 128>;
  constexpr int D = M::D, NCH = M::NCH, RS = M::RS, SL = M::SL, NT = 256;
  constexpr long long kWait = 1ll << 31;
  constexpr uint32_t kId1 = tc::idesc_bf16(128, kC, 0, 0);  // [K; Q] K^T: both K-major
  constexpr uint32_t kId2 = tc::idesc_bf16(128, D, 0, 1);   // [T1; T2] (K-major) x K | V (MN-major)
  extern __shared__ __align__(16) unsigned char smem[];
  __nv_bfloat16* sRawT = reinterpret_cast<__nv_bfloat16*>(smem);  // [kC + 3][RS]
  float* sL = reinterpret_cast<float*>(smem + M::l);
  float* sTmp = reinterpret_cast<float*>(smem + M::tmp);
  unsigned char* sKi = smem + M::k;
  unsigned char* sQi = smem + M::q;
  float* sG = reinterpret_cast<float*>(smem + M::vec);
  float* sBeta = sG + kC;
  float* sRaw = sBeta + kC;
  float* sEG = sRaw + kC;   // e^{G_i}
  float* sW1 = sEG + kC;    // beta_i e^{G_i} / |k_i|: the columns of T1
  float* sEGL = sW1 + kC;   // e^{G_last - G_i}
  float* sIq = sEGL + kC;   // |q_i|^2, then scale / |q_i|
  float* sIk = sIq + kC;    // |k_i|^2, then 1 / |k_i|
  float* sG2 = sIk + kC;    // G_i log2 e
  float* sIk2 = sG2 + kC;   // [kC] (1 / |k_j|, G_j log2 e) pairs
  __nv_bfloat16* sCw = reinterpret_cast<__nv_bfloat16*>(smem + M::cw);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + M::bar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + M::slot);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = blockIdx.x;
  const int bh = blockIdx.y, b = bh / a.HV, hv = bh % a.HV, h = hv / (a.HV / a.H);
  const int key_dim = a.H * D, conv_dim = 2 * key_dim + a.HV * D;
  const int t0 = c * kC;
  auto chan = [&](int lc) {  // head-local channel -> projection column
    return lc < D ? h * D + lc : (lc < 2 * D ? key_dim + h * D + (lc - D) : 2 * key_dim + hv * D + (lc - 2 * D));
  };
  int64_t seq0;
  int L;
  seq_of(a, b, seq0, L);
  if (t0 >= L) return;  // past this request's last chunk (varlen): the whole CTA, before any barrier
  const __nv_bfloat16* prow0 = a.proj + seq0 * a.ld_proj;
  unsigned char* blk = a.blocks + (int64_t(bh) * a.nc + c) * CB::bytes;

  // ---- stage the raw projection tile (tokens t0-3 .. t0+63, zero outside [0, L)) -----
  {
    constexpr int CPR = NCH / 8, GRP = NT / CPR;
    if (tid < GRP * CPR) {
      const int lc = (tid % CPR) * 8;
      const __nv_bfloat16* src = prow0 + chan(lc);
      __nv_bfloat16* dst = sRawT + lc;
      for (int r = tid / CPR; r < kC + 3; r += GRP) {
        const int t = t0 - 3 + r;
        if (t >= 0 && t < L) cp_async16(dst + r * RS, src + int64_t(t) * a.ld_proj);
        else *reinterpret_cast<uint4*>(dst + r * RS) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    for (int i = tid; i < NCH / 2; i += NT) cp_async16(sCw + i * 8, a.conv_w + int64_t(chan(2 * i)) * 4);
  }
  cp_async_commit();
  float gb = 0.f, ga = 0.f;  // gate inputs of token t0 + tid
  if (tid < kC && t0 + tid < L) {
    const __nv_bfloat16* pr = prow0 + int64_t(t0 + tid) * a.ld_proj + conv_dim + int64_t(a.HV) * D;
    gb = __bfloat162float(pr[hv]);
    ga = __bfloat162float(pr[a.HV + hv]);
  }
  if (warp == 0) tc::tmem_alloc(tslot, 256);
  if (tid == 0) {
    tc::mbar_init(mbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  cp_async_wait<0>();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t sb = smem_u32(smem);

  // ---- conv + SiLU into the k | q | v images; squared norms of q and k rows ---------
  // 48 groups of 8 channels x 16 segments of 4 tokens = 3 items a thread; a half-warp's
  // 16 items are the 16 groups of one of q / k / v for one segment
  {
    constexpr int NG = NCH / 8, SEG = 4;
    static_assert(NG * (kC / SEG) == 3 * NT, "every thread takes the same number of items");
    float ssq_all[3][SEG];  // per item: the squared norms' partial sums, reduced after the loop
#pragma unroll
    for (int it = 0; it < 3; ++it) {
      const int item = tid + it * NT;
      const int grp = item % NG, seg = item / NG;
      const int lc = grp * 8, part = grp / (D / 8);  // 0: q, 1: k, 2: v
      float2 w2[4][4];
      {
        const uint4* wp = reinterpret_cast<const uint4*>(sCw + lc * 4);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint4 raw = wp[u];
          const float2 c0a = bf2f(raw.x), c0b = bf2f(raw.y), c1a = bf2f(raw.z), c1b = bf2f(raw.w);
          w2[u][0] = make_float2(c0a.x, c1a.x);
          w2[u][1] = make_float2(c0a.y, c1a.y);
          w2[u][2] = make_float2(c0b.x, c1b.x);
          w2[u][3] = make_float2(c0b.y, c1b.y);
        }
      }
      auto row4 = [&](int r, float2 (&v)[4]) {
        const uint4 u = *reinterpret_cast<const uint4*>(sRawT + r * RS + lc);
        v[0] = bf2f(u.x);
        v[1] = bf2f(u.y);
        v[2] = bf2f(u.z);
        v[3] = bf2f(u.w);
      };
      const int r0 = seg * SEG;
      float2 win[3][4];
      row4(r0, win[0]);
      row4(r0 + 1, win[1]);
      row4(r0 + 2, win[2]);
      unsigned char* img = smem + (part == 0 ? M::q : (part == 1 ? M::k : M::v));
      const int ch = grp % (D / 8);
#pragma unroll
      for (int rr = 0; rr < SEG; ++rr) {
        const int r = r0 + rr;
        float2 x[4];
        row4(r + 3, x);
        uint4 u = make_uint4(0u, 0u, 0u, 0u);
        float2 s2 = make_float2(0.f, 0.f);
        if (t0 + r < L) {
          uint32_t* uw = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
          for (int pp = 0; pp < 4; ++pp) {
            float2 acc = mul2(win[0][pp], w2[pp][0]);
            acc = fma2(win[1][pp], w2[pp][1], acc);
            acc = fma2(win[2][pp], w2[pp][2], acc);
            acc = fma2(x[pp], w2[pp][3], acc);
            uw[pp] = bf2_pack_f2(silu2(acc));
            const float2 o = bf2f(uw[pp]);
            s2 = fma2(o, o, s2);
          }
        }
        ssq_all[it][rr] = s2.x + s2.y;
        *reinterpret_cast<uint4*>(img + M::img_off(r, ch)) = u;
#pragma unroll
        for (int pp = 0; pp < 4; ++pp) {
          win[0][pp] = win[1][pp];
          win[1][pp] = win[2][pp];
          win[2][pp] = x[pp];
        }
      }
    }
    // half-warp sums (a half-warp's 16 items of one item slot are the 16 groups of one of
    // q / k / v for one segment): 12 independent shuffle chains
#pragma unroll
    for (int it = 0; it < 3; ++it)
#pragma unroll
      for (int rr = 0; rr < SEG; ++rr)
#pragma unroll
        for (int m = 1; m < 16; m <<= 1) ssq_all[it][rr] += __shfl_xor_sync(0xffffffffu, ssq_all[it][rr], m);
    if ((lane & 15) == 0)
#pragma unroll
      for (int it = 0; it < 3; ++it) {
        const int item = tid + it * NT, grp = item % NG, part = grp / (D / 8), r0 = (item / NG) * SEG;
        if (part < 2)
#pragma unroll
          for (int rr = 0; rr < SEG; ++rr) (part == 0 ? sIq : sIk)[r0 + rr] = ssq_all[it][rr];
      }
  }
  if (t0 + kC >= L) {  // last chunk: conv state = pre-conv columns of tokens L-4 .. L-1
    for (int lc = tid; lc < NCH; lc += NT) {
      __nv_bfloat16 s4[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) s4[j] = sRawT[(L - 1 - t0 + j) * RS + lc];
      *reinterpret_cast<uint2*>(a.conv_state + (int64_t(b) * conv_dim + chan(lc)) * 4) = *reinterpret_cast<uint2*>(s4);
    }
  }
  if (tid < kC) {  // gates
    float g = 0.f, be = 0.f;
    if (t0 + tid < L) {
      be = bf16r(sigmoid_f(gb));
      g = -expf(a.a_log[hv]) * softplus_f(ga + a.dt_bias[hv]);
    }
    sRaw[tid] = g;
    sBeta[tid] = be;
  }
  tc::fence_async_smem();  // the images -> tensor cores
  tc::fence_before();
  __syncthreads();
  tc::fence_after();

  // ---- MMA1 (one thread) while the others finish norms, gates and decays --------------
  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < D / 16; ++s) {
      const uint64_t d = tc::smem_desc(sb + M::k + s * 2 * M::CST, M::CST, M::GST);
      tc::mma_bf16(tmem, d, d, kId1, s > 0);
    }
    tc::commit(mbar);
  }
  if (tid < 2 * kC) {
    const int r = tid & (kC - 1);
    if (tid < kC) sIq[r] = a.scale / sqrtf(sIq[r] + 1e-6f);
    else sIk[r] = 1.0f / sqrtf(sIk[r] + 1e-6f);
  } else if (warp == 4) {  // in-chunk cumulative log decay (warp scan over 64 values)
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
  }
  __syncthreads();
  if (tid < kC) {
    const float e = __expf(sG[tid]);
    sEG[tid] = e;
    sW1[tid] = sBeta[tid] * e * sIk[tid];
    sEGL[tid] = __expf(sG[kC - 1] - sG[tid]);
    sG2[tid] = sG[tid] * 1.4426950408889634f;
    reinterpret_cast<float2*>(sIk2)[tid] = make_float2(sIk[tid], sG2[tid]);
  }
  __syncthreads();

  // ---- MMA1 epilogue: L = strictly-lower(beta_i K K^T o e^{G_i - G_j}) (fp32, shared),
  //      Aqk = lower(Q K^T o e^{G_i - G_j}) (bf16, to the block), a thread per row --------
  bool ok = tc::mbar_wait(mbar, 0, kWait);
  tc::fence_after();
  {
    const int quad = warp & 3, hc = warp >> 2;  // TMEM lanes 32 quad .., columns 32 hc ..
    const int i = (quad * 32 + lane) & (kC - 1);
    // rows 0..31 against columns 32..63 lie above the diagonal: zeros, no TMEM read
    const bool upper = (quad & 1) == 0 && hc == 1;
    uint32_t v[32];
    if (!upper) {
      tc::ld32(tc::taddr(tmem, quad * 32, hc * 32), v);
      tc::wait_ld();
    }
    const float Gi = sG2[i];
    const float2* cf = reinterpret_cast<const float2*>(sIk2) + hc * 32;  // (1 / |k_j|, G_j log2 e)
    if (quad < 2) {  // K K^T row i
      const float f = sBeta[i] * sIk[i];
      if (upper) {
#pragma unroll
        for (int e = 0; e < 32; ++e) sL[i * SL + hc * 32 + e] = 0.f;
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int j = hc * 32 + e;
          const float2 c = cf[e];
          sL[i * SL + j] = j < i ? f * c.x * __uint_as_float(v[e]) * fast_ex2(Gi - c.y) : 0.f;
        }
      }
    } else {  // Q K^T row i -> the block's 64-wide K-major core tile
      const float f = sIq[i];
      uint32_t pk[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int j = hc * 32 + 2 * e;
        const float2 c0 = cf[2 * e], c1 = cf[2 * e + 1];
        const float x0 = !upper && j <= i ? f * c0.x * __uint_as_float(v[2 * e]) * fast_ex2(Gi - c0.y) : 0.f;
        const float x1 =
            !upper && j + 1 <= i ? f * c1.x * __uint_as_float(v[2 * e + 1]) * fast_ex2(Gi - c1.y) : 0.f;
        pk[e] = bf2_pack(x0, x1);
      }
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4)
        *reinterpret_cast<uint4*>(blk + CB::aqk + (i >> 3) * 1024 + (hc * 4 + q4) * 128 + (i & 7) * 16) =
            make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
    }
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();

  if (warp < 4) {
    // ---- T = (I + L)^-1 (warps 0-3, named barrier 1) ---------------------------------
    if (tid < kC) {  // diagonal 16x16 blocks: lane (block, column j) forward-substitutes column j
      const int d0 = (tid >> 4) * 16, j = tid & 15;
      const float* Lb = sL + d0 * SL + d0;
      float t[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float acc = 0.f;
#pragma unroll
        for (int m = 0; m < i; ++m) acc = fmaf(Lb[i * SL + m], t[m], acc);
        t[i] = i < j ? 0.f : (i == j ? 1.f : -acc);
      }
      __syncwarp();
#pragma unroll
      for (int i = 1; i < 16; ++i)
        if (i > j) sL[(d0 + i) * SL + d0 + j] = t[i];
    }
    named_bar(1, 128);
    if (tid < kC) sL[tid * SL + tid] = 1.f;
    named_bar(1, 128);
    {  // level 1 (16x16 blocks, TF32): T_10 = -T_11 (L_10 T_00), T_32 = -T_33 (L_32 T_22)
      const int bp = warp >> 1, nc8 = warp & 1;
      const int r0 = 16 + 32 * bp, c0 = 32 * bp;
      float acc[1][4];
      zero_acc<1>(acc);
      warp_mma_tf32<16, 1>(acc, sL + r0 * SL + c0, SL, sL + c0 * SL + c0 + nc8 * 8, SL);
      store_acc<1>(sTmp + bp * 16 * 33 + nc8 * 8, 33, acc, 1.f);
      named_bar(1, 128);
      zero_acc<1>(acc);
      warp_mma_tf32<16, 1>(acc, sL + r0 * SL + r0, SL, sTmp + bp * 16 * 33 + nc8 * 8, 33);
      named_bar(1, 128);
      store_acc<1>(sL + r0 * SL + c0 + nc8 * 8, SL, acc, -1.f);
    }
    named_bar(1, 128);
    {  // level 2 (32x32 blocks): T_[2:4][0:2] = -T_D (C T_A) with C = L[32:64, 0:32]
      const int mt = warp >> 1, nh = warp & 1;
      float acc[2][4];
      zero_acc<2>(acc);
      warp_mma_tf32<32, 2>(acc, sL + (32 + mt * 16) * SL, SL, sL + nh * 16, SL);
      store_acc<2>(sTmp + mt * 16 * 33 + nh * 16, 33, acc, 1.f);
      named_bar(1, 128);
      zero_acc<2>(acc);
      warp_mma_tf32<32, 2>(acc, sL + (32 + mt * 16) * SL + 32, SL, sTmp + nh * 16, 33);
      named_bar(1, 128);
      store_acc<2>(sL + (32 + mt * 16) * SL + nh * 16, SL, acc, -1.f);
    }
  } else {
    // ---- warps 4-7: Q' = e^{G_i} scale q_i / |q_i| and K' = e^{G_last - G_i} k_i / |k_i| -------
    const int t = tid - 128, i = t & (kC - 1);
    const bool isk = t >= kC;
    const unsigned char* src = isk ? sKi : sQi;
    unsigned char* dst = blk + (isk ? CB::kp : CB::q) + (i >> 3) * 2048 + (i & 7) * 16;
    const float f = isk ? sEGL[i] * sIk[i] : sEG[i] * sIq[i];
#pragma unroll 4
    for (int ch = 0; ch < D / 8; ++ch) {
      uint4 raw = *reinterpret_cast<const uint4*>(src + M::img_off(i, ch));
      uint32_t* w = reinterpret_cast<uint32_t*>(&raw);
#pragma unroll
      for (int e = 0; e < 4; ++e) w[e] = bf2_pack_f2(mul2(bf2f(w[e]), make_float2(f, f)));
      *reinterpret_cast<uint4*>(dst + ch * 128) = raw;
    }
  }
  __syncthreads();

  // ---- [T1; T2] as a K-major core tile (rows i, K = tokens j) ---------------------------
  for (int u = tid; u < 2 * kC * (kC / 8); u += NT) {
    const int i = (u & 7) | ((u >> 6) << 3), jc = (u >> 3) & 7;
    const int ti = i & (kC - 1);
    const float* fac = i >= kC ? sBeta : sW1;
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = jc * 8 + 2 * e;
      const float v0 = ti >= j ? sL[ti * SL + j] : 0.f;
      const float v1 = ti >= j + 1 ? sL[ti * SL + j + 1] : 0.f;
      w[e] = bf2_pack(v0 * fac[j], v1 * fac[j + 1]);
    }
    *reinterpret_cast<uint4*>(smem + M::t12 + (i >> 3) * 1024 + jc * 128 + (i & 7) * 16) =
        make_uint4(w[0], w[1], w[2], w[3]);
  }
  tc::fence_async_smem();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  if (tid == 0) {  // MMA2: [T1; T2] K -> columns 0..127, [T1; T2] V -> columns 128..255
#pragma unroll
    for (int s = 0; s < kC / 16; ++s) {
      const uint64_t ad = tc::smem_desc(sb + M::t12 + s * 256, 128, 1024);
      tc::mma_bf16(tmem, ad, tc::smem_desc(sb + M::k + s * 2 * M::GST, M::GST, M::CST), kId2, s > 0);
      tc::mma_bf16(tmem + 128, ad, tc::smem_desc(sb + M::v + s * 2 * M::GST, M::GST, M::CST), kId2, s > 0);
    }
    tc::commit(mbar);
  }
  if (tid < kC / 4) reinterpret_cast<float4*>(blk + CB::g)[tid] = reinterpret_cast<const float4*>(sG)[tid];
  ok = tc::mbar_wait(mbar, 1, kWait) && ok;
  tc::fence_after();
  {  // W = rows 0..63 of [T1; T2] K (quadrants 0, 1); U = rows 64..127 of [T1; T2] V (2, 3)
    const int quad = warp & 3, hc = warp >> 2;
    const int i = (quad * 32 + lane) & (kC - 1);
    const bool isu = quad >= 2;
#pragma unroll
    for (int piece = 0; piece < 2; ++piece) {
      uint32_t v[32];
      tc::ld32(tc::taddr(tmem, quad * 32, (isu ? 128 : 0) + hc * 64 + piece * 32), v);
      tc::wait_ld();
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const int ch = hc * 8 + piece * 4 + q4;
        uint4 res;
        uint32_t* rw = reinterpret_cast<uint32_t*>(&res);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          rw[e] = bf2_pack(__uint_as_float(v[q4 * 8 + 2 * e]), __uint_as_float(v[q4 * 8 + 2 * e + 1]));
        if (isu) *reinterpret_cast<uint4*>(blk + CB::u + i * 256 + ((ch ^ (i & 7)) * 16)) = res;
        else *reinterpret_cast<uint4*>(blk + CB::w + (i >> 3) * 2048 + ch * 128 + (i & 7) * 16) = res;
      }
    }
  }
  if (!ok && lane == 0) atomicOr(a.status, 1u);  // an MMA completion wait timed out
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::tmem_free(tmem, 256);
  }
}

// ---------------------------------------------------------------------------
// scan
// ---------------------------------------------------------------------------
template <int DK, int DV>
struct ScanSmem {
  static constexpr int SQ = DK + 8, SV = DV + 8, ST = kC + 8;
  // one pipeline stage = one chunk block with padded rows
  static constexpr size_t q = 0;
  static constexpr size_t kp = q + size_t(kC) * SQ * 2;
  static constexpr size_t w = kp + size_t(kC) * SQ * 2;
  static constexpr size_t u = w + size_t(kC) * SQ * 2;
  static constexpr size_t aqk = u + size_t(kC) * SV * 2;
  static constexpr size_t g = aqk + size_t(kC) * ST * 2;
  static constexpr size_t stage = g + size_t(kC) * 4;
  static constexpr size_t s = 2 * stage;                  // S (bf16) [DK][SV]
  static constexpr size_t vn = s + size_t(DK) * SV * 2;   // Vn [kC][SV]
  static constexpr size_t ss = vn + size_t(kC) * SV * 2;  // row sums of squares [kC][2]
  static constexpr size_t bytes = ss + size_t(kC) * 2 * 4;
  static_assert(stage % 16 == 0 && s % 16 == 0 && vn % 16 == 0, "alignment");
};

// Copy a dense [rows][COLS] bf16 tile into padded shared rows with cp.async.
template <int COLS>
__device__ __forceinline__ void stage_tile(__nv_bfloat16* dst, int lds, const __nv_bfloat16* src, int tid) {
  constexpr int CH = COLS / 8;
  for (int i = tid; i < kC * CH; i += 256) {
    const int r = i / CH, c = (i % CH) * 8;
    cp_async16(dst + r * lds + c, src + r * COLS + c);
  }
}

template <int DK, int DV>
__global__ void __launch_bounds__(256, 1) gdn_scan_kernel(const SplitArgs a) {
  using M = ScanSmem<DK, DV>;
  using CB = ChunkBlock<DK, DV>;
  constexpr int SQ = M::SQ, SV = M::SV, ST = M::ST;
  constexpr int NT = DV / 16;     // n8 tiles of one column half
  constexpr int SROWS = DK / 16;  // warps holding S rows
  static_assert(SROWS <= 8, "one S m-tile per warp");
  extern __shared__ __align__(16) unsigned char smem[];
  __nv_bfloat16* sS = reinterpret_cast<__nv_bfloat16*>(smem + M::s);
  __nv_bfloat16* sVn = reinterpret_cast<__nv_bfloat16*>(smem + M::vn);
  float* sSS = reinterpret_cast<float*>(smem + M::ss);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bh = blockIdx.x, b = bh / a.HV, hv = bh % a.HV;
  const int g8 = lane >> 2, tq = lane & 3;
  const int mt = warp & 3, nh = warp >> 2;  // output tile: rows mt*16.., columns nh*DV/2..
  const int i0 = mt * 16 + g8, i1 = i0 + 8;
  const int conv_dim = 2 * a.H * DK + a.HV * DV;
  const unsigned char* blocks = a.blocks + int64_t(bh) * a.nc * CB::bytes;

  auto load_block = [&](int c, int st) {
    const unsigned char* src = blocks + int64_t(c) * CB::bytes;
    unsigned char* dst = smem + st * M::stage;
    stage_tile<DK>(reinterpret_cast<__nv_bfloat16*>(dst + M::q), SQ, reinterpret_cast<const __nv_bfloat16*>(src + CB::q), tid);
    stage_tile<DK>(reinterpret_cast<__nv_bfloat16*>(dst + M::kp), SQ, reinterpret_cast<const __nv_bfloat16*>(src + CB::kp), tid);
    stage_tile<DK>(reinterpret_cast<__nv_bfloat16*>(dst + M::w), SQ, reinterpret_cast<const __nv_bfloat16*>(src + CB::w), tid);
    stage_tile<DV>(reinterpret_cast<__nv_bfloat16*>(dst + M::u), SV, reinterpret_cast<const __nv_bfloat16*>(src + CB::u), tid);
    stage_tile<kC>(reinterpret_cast<__nv_bfloat16*>(dst + M::aqk), ST, reinterpret_cast<const __nv_bfloat16*>(src + CB::aqk), tid);
    if (tid < kC / 4) cp_async16(dst + M::g + tid * 16, src + CB::g + tid * 16);
  };

  float S[DV / 8][4];
  zero_acc<DV / 8>(S);
  for (int i = tid; i < DK * SV; i += 256) sS[i] = __float2bfloat16_rn(0.f);
  load_block(0, 0);
  cp_async_commit();
  for (int c = 0; c < a.nc; ++c) {
    const int st = c & 1;
    cp_async_wait<0>();
    __syncthreads();  // block c landed; every warp is past chunk c - 1
    if (c + 1 < a.nc) {
      load_block(c + 1, st ^ 1);
      cp_async_commit();
    }
    const unsigned char* sb = smem + st * M::stage;
    const __nv_bfloat16* sQ = reinterpret_cast<const __nv_bfloat16*>(sb + M::q);
    const __nv_bfloat16* sKp = reinterpret_cast<const __nv_bfloat16*>(sb + M::kp);
    const __nv_bfloat16* sW = reinterpret_cast<const __nv_bfloat16*>(sb + M::w);
    const __nv_bfloat16* sU = reinterpret_cast<const __nv_bfloat16*>(sb + M::u);
    const __nv_bfloat16* sA = reinterpret_cast<const __nv_bfloat16*>(sb + M::aqk);
    const float* sG = reinterpret_cast<const float*>(sb + M::g);
    // [W; Q'] S for this warp's tile; Vn = U - W S -> sVn, O = Q' S (= e^G Q S)
    float pw[NT][4], o[NT][4];
    zero_acc<NT>(pw);
    zero_acc<NT>(o);
    warp_mma<DK, NT, false, true>(pw, sW, SQ, mt * 16, 0, sS, SV, 0, nh * (DV / 2));
    warp_mma<DK, NT, false, true>(o, sQ, SQ, mt * 16, 0, sS, SV, 0, nh * (DV / 2));
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int col = nh * (DV / 2) + j * 8 + tq * 2;
      const __nv_bfloat162 u0 = *reinterpret_cast<const __nv_bfloat162*>(sU + i0 * SV + col);
      const __nv_bfloat162 u1 = *reinterpret_cast<const __nv_bfloat162*>(sU + i1 * SV + col);
      *reinterpret_cast<__nv_bfloat162*>(sVn + i0 * SV + col) =
          __floats2bfloat162_rn(__low2float(u0) - pw[j][0], __high2float(u0) - pw[j][1]);
      *reinterpret_cast<__nv_bfloat162*>(sVn + i1 * SV + col) =
          __floats2bfloat162_rn(__low2float(u1) - pw[j][2], __high2float(u1) - pw[j][3]);
    }
    __syncthreads();  // Vn complete; every read of sS for this chunk is done
    // S <- e^{G_last} S + K'^T Vn;  O += Aqk Vn
    if (warp < SROWS) {
      const float dl = __expf(sG[kC - 1]);
#pragma unroll
      for (int j = 0; j < DV / 8; ++j) {
        S[j][0] *= dl; S[j][1] *= dl; S[j][2] *= dl; S[j][3] *= dl;
      }
      warp_mma<kC, DV / 8, true, true>(S, sKp, SQ, warp * 16, 0, sVn, SV, 0, 0);
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
      sSS[i0 * 2 + nh] = ss0;
      sSS[i1 * 2 + nh] = ss1;
    }
    if (warp < SROWS) {
#pragma unroll
      for (int j = 0; j < DV / 8; ++j) {
        const int r0 = warp * 16 + g8, col = j * 8 + tq * 2;
        *reinterpret_cast<__nv_bfloat162*>(sS + r0 * SV + col) = __floats2bfloat162_rn(S[j][0], S[j][1]);
        *reinterpret_cast<__nv_bfloat162*>(sS + (r0 + 8) * SV + col) = __floats2bfloat162_rn(S[j][2], S[j][3]);
      }
    }
    __syncthreads();  // row norms complete
    // gated RMSNorm of O, times SiLU(z), to the layer output
    const int nvalid = min(kC, a.L - c * kC);
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int i = hr ? i1 : i0;
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

// ---------------------------------------------------------------------------
// scan on the 5th-generation tensor cores (DK = DV = 128): S and the chunk
// products live in tensor memory.  Warps 0-7: warp w reads TMEM lane quadrant
// w % 4, columns [64 (w / 4), +64).
//   TMEM columns [0, 128): S (lane = key row);  [128, 256): P / O (lane = row)
//   MMA1  P  = [W; Q'] S          (M 128 = 64 W rows + 64 Q' rows, K = 128)
//   V warps (quadrants 0, 1): Vn = U - W S -> shared memory (MN-major B operand)
//   MMA2  S (+)= K'^T Vn          (M = 128 key rows, K = 64 tokens)
//   MMA3  P += [any; Aqk] Vn      (rows 64..127 become O; rows 0..63 land in the
//                                  consumed W lanes, so no zero rows are staged)
//   warps 0-7: S -> BF16 copy (next MMA1's B operand), then S *= e^{G_last} of
//   the next chunk; O warps (quadrants 2, 3) stash BF16 O and its row sums of
//   squares in shared memory, and warps 8-11 run the gated RMSNorm on the stash
//   during the next chunk's MMA1 -> Vn -> MMA2/3.
// The MMA issuer is thread 0 (a V warp).  mbarriers: bar1 (MMA1) and bar2
// (MMA2/3) complete once per chunk, so parity c & 1 names the chunk's phase.
// ---------------------------------------------------------------------------
struct TcScan {
  static constexpr int D = 128;
  using CB = ChunkBlock<128, 128>;
  // one stage = the chunk block's image up to G (one bulk copy): w | q | kp | aqk | u
  static constexpr size_t a1 = CB::w;                      // [W; Q'] K-major core tile, 128 rows x K 128
  static constexpr size_t a2 = CB::kp;                     // K' MN-major, M 128 (keys) x K 64 (tokens)
  // [any; Aqk] K-major, 128 rows x K 64: rows 0..63 are K' bytes, whose products land in
  // the TMEM lanes of the W rows, already consumed when that MMA runs
  static constexpr size_t a3 = CB::aqk - size_t(kC) * kC * 2;
  static constexpr size_t u = CB::u;                       // U: 256-byte rows, XOR-swizzled chunks
  static constexpr size_t stage = CB::g;                   // bytes of a stage (= of its copy)
  static constexpr size_t b1 = 2 * stage;                  // S (bf16) MN-major, K 128 (keys) x N 128
  static constexpr size_t b2 = b1 + size_t(D) * D * 2;     // Vn MN-major, K 64 (tokens) x N 128
  static constexpr size_t ost = b2 + size_t(kC) * D * 2;   // O stash [64][128] bf16, 16-byte chunks XOR (row % 8)
  static constexpr int kGMax = 1024;                       // chunks whose last decay is preloaded
  static constexpr size_t gl = ost + size_t(kC) * D * 2;   // [kGMax] fp32 G_last of every chunk
  static constexpr size_t bar = gl + size_t(kGMax) * 4;    // mbarriers: MMA1, MMA2/3, stage 0, stage 1
  static constexpr size_t slot = bar + 4 * 8;              // TMEM base address
  static constexpr size_t nw = slot + 16;                  // [128] fp32 norm weight
  static constexpr size_t nss = nw + size_t(D) * 4;        // [64][2] fp32 O row-half sums of squares
  static constexpr size_t bytes = nss + size_t(kC) * 2 * 4;
  static_assert(a1 == 0 && CB::q == size_t(kC) * D * 2 && stage % 16 == 0 && bar % 8 == 0 && nw % 16 == 0,
                "stage image");
  static_assert(bytes <= 232448, "shared memory");
  // core-matrix byte offset of (row, 16-byte chunk) in 128-wide tiles (SBO 2048, LBO 128)
  __device__ static uint32_t off16(int r, int ch) { return (r >> 3) * 2048 + ch * 128 + (r & 7) * 16; }
  // U row r, chunk ch: rows of 256 bytes, chunk index XOR (r % 8); the O stash likewise
  __device__ static uint32_t offu(int r, int ch) { return r * 256 + ((ch ^ (r & 7)) * 16); }
};

// Gated RMSNorm of one O row half (64 columns, BF16 in `ob`) of the tensor-core scan:
//   out = bf16( bf16(w * bf16(o * rsqrt(mean(o^2) + eps))) * silu(z) )
// (Qwen3_5RMSNormGated, modeling_qwen3_5.py:175-190; o is the BF16 gated_delta output),
// with ss the sum of squares over the whole row.
__device__ __forceinline__ void gated_norm_half(const uint32_t (&ob)[32], const uint4 (&zq)[8], const float* nw,
                                                float ss, float eps, uint4* dst) {
  const float inv = 1.0f / sqrtf(ss / 128.f + eps);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 w0 = *reinterpret_cast<const float4*>(nw + q * 8);
    const float4 w1 = *reinterpret_cast<const float4*>(nw + q * 8 + 4);
    const float2 w[4] = {make_float2(w0.x, w0.y), make_float2(w0.z, w0.w), make_float2(w1.x, w1.y),
                         make_float2(w1.z, w1.w)};
    const uint32_t zw[4] = {zq[q].x, zq[q].y, zq[q].z, zq[q].w};
    uint32_t res[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float2 n = bf2f(bf2_pack_f2(mul2(bf2f(ob[q * 4 + p]), make_float2(inv, inv))));  // bf16(o * inv)
      const float2 h = bf2f(bf2_pack_f2(mul2(w[p], n)));                                       // bf16(w * .)
      res[p] = bf2_pack_f2(mul2(h, silu2(bf2f(zw[p]))));
    }
    dst[q] = make_uint4(res[0], res[1], res[2], res[3]);
  }
}

__device__ __forceinline__ void named_arrive(int id, int n) {
  asm volatile("bar.arrive %0, %1;\n" ::"r"(id), "r"(n) : "memory");
}

// Sequential chunk scan, S in TMEM (12 warps).  Warps 0-7: quadrants 0, 1 (lanes 0-63) hold
// the W rows of P = [W; Q'] S and compute Vn = U - W S; quadrants 2, 3 (lanes 64-127) hold
// O = Q' S + Aqk Vn, staged as BF16 with its row sums of squares in shared memory; all eight
// carry S.  Warps 8-11 apply the gated RMSNorm to the stashed O of chunk c - 1 while chunk c
// runs (named barrier 3 hands the stash back before chunk c's O overwrites it).
__global__ void __launch_bounds__(384, 1) gdn_scan_tc_kernel(const SplitArgs a) {
  using M = TcScan;
  using CB = ChunkBlock<128, 128>;
  constexpr int D = 128, NTH = 384;
  constexpr long long kWait = 1ll << 31;  // ~1 s of SM clocks per MMA wait
  constexpr uint32_t kId1 = tc::idesc_bf16(128, 128, 0, 1);  // K-major A, MN-major B
  constexpr uint32_t kId2 = tc::idesc_bf16(128, 128, 1, 1);  // MN-major A and B
  extern __shared__ __align__(16) unsigned char smem[];
  uint64_t* bar1 = reinterpret_cast<uint64_t*>(smem + M::bar);  // MMA1 commits
  uint64_t* bar2 = bar1 + 1;                                       // MMA2/3 commits
  uint64_t* ldbar = bar1 + 2;                                      // stage loads [2]
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + M::slot);
  float* sNw = reinterpret_cast<float*>(smem + M::nw);
  float* sNss = reinterpret_cast<float*>(smem + M::nss);
  float* sGL = reinterpret_cast<float*>(smem + M::gl);  // G_last of each chunk: off the per-chunk critical path
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool nwarp = warp >= 8;  // gated RMSNorm warps
  const int quad = warp & 3, half = (warp >> 2) & 1;
  const int row = quad * 32 + lane;  // TMEM lane of this thread (warps 0-7)
  const bool vwarp = !nwarp && quad < 2;
  const bool issuer = tid == 0;
  const int bh = blockIdx.x, b = bh / a.HV, hv = bh % a.HV;
  const unsigned char* blocks = a.blocks + int64_t(bh) * a.nc * CB::bytes;  // row of a.nc (longest) chunks
  const uint32_t sbase = smem_u32(smem);
  int64_t seq0;
  int L;
  seq_of(a, b, seq0, L);
  const int nc = (L + kC - 1) / kC;  // this request's chunks

  int ld_issued[2] = {0, 0};  // stage loads issued (issuer thread)
  auto load_block = [&](int c, int st) {  // issuer: chunk block c (its shared-memory image) -> stage st
    tc::mbar_expect_tx(ldbar + st, uint32_t(M::stage));
    tc::bulk_g2s(smem + st * M::stage, blocks + int64_t(c) * CB::bytes, uint32_t(M::stage), ldbar + st);
    ++ld_issued[st];
  };

  // S = 0 (bf16 copy), norm weight, G_last, barriers, TMEM
  for (int i = tid; i < D * D * 2 / 16; i += NTH) reinterpret_cast<uint4*>(smem + M::b1)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) tc::mbar_init(bar1 + i, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 0) tc::tmem_alloc(slot, 256);
  if (tid < D) sNw[tid] = a.norm_w[tid];
  for (int i = tid; i < nc && i < M::kGMax; i += NTH)
    sGL[i] = *reinterpret_cast<const float*>(blocks + int64_t(i) * CB::bytes + CB::g + (kC - 1) * 4);
  tc::fence_async_smem();  // zeroed S copy -> tensor cores
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  if (issuer) load_block(0, 0);
  const uint32_t tmem = *slot;
  const uint32_t lane_off = uint32_t(quad * 32) << 16;
  const uint32_t tS = tmem + lane_off + half * 64, tP = tmem + 128 + lane_off + half * 64;
  bool ok = true;

  // norm warps: thread (token nr of the chunk, column half nh)
  const int conv_dim = 2 * a.H * D + a.HV * D;
  const int nr = (tid - 256) & (kC - 1), nh = ((tid - 256) >> 6) & 1;
  auto norm_chunk = [&](int c, bool hand_back) {  // gated RMSNorm of chunk c's stashed O rows
    uint32_t ob[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint4 v = *reinterpret_cast<const uint4*>(smem + M::ost + M::offu(nr, nh * 8 + q));
      ob[4 * q] = v.x;
      ob[4 * q + 1] = v.y;
      ob[4 * q + 2] = v.z;
      ob[4 * q + 3] = v.w;
    }
    const float ss = sNss[nr * 2] + sNss[nr * 2 + 1];
    if (hand_back) named_arrive(3, 256);  // the stash may take chunk c + 1's O
    const int64_t t = int64_t(c) * kC + nr;
    if (t >= L) return;
    const uint4* zp = reinterpret_cast<const uint4*>(a.proj + (seq0 + t) * a.ld_proj + conv_dim + hv * D + nh * 64);
    uint4 zq[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) zq[q] = __ldg(zp + q);
    gated_norm_half(ob, zq, sNw + nh * 64, ss, a.eps,
                    reinterpret_cast<uint4*>(a.out + (seq0 + t) * a.ld_out + hv * D + nh * 64));
  };

  for (int c = 0; c < nc; ++c) {
    const int st = c & 1;
    const uint32_t par = uint32_t(c) & 1u;
    const unsigned char* sb = smem + st * M::stage;
    const uint32_t sbu = sbase + st * M::stage;
    ok = tc::mbar_wait(ldbar + st, uint32_t(c >> 1) & 1u, kWait) && ok;  // block c staged
    tc::fence_async_smem();
    tc::fence_before();
    ok = __syncthreads_and(ok);  // chunk c-1's S copy, TMEM traffic and stage reads done
    if (!ok) break;
    tc::fence_after();
    if (nwarp) {
      if (c > 0) norm_chunk(c - 1, true);
      continue;
    }
    const float gl_next =
        c + 1 >= nc ? 0.f
                    : (c + 1 < M::kGMax ? sGL[c + 1]
                                        : *reinterpret_cast<const float*>(blocks + int64_t(c + 1) * CB::bytes + CB::g +
                                                                          (kC - 1) * 4));
    if (vwarp) {
      if (issuer) {  // MMA1: P = [W; Q'] S
#pragma unroll
        for (int s = 0; s < 8; ++s)
          tc::mma_bf16(tmem + 128, tc::smem_desc(sbu + M::a1 + s * 256, 128, 2048),
                       tc::smem_desc(sbase + M::b1 + s * 4096, 2048, 128), kId1, s > 0);
        tc::commit(bar1);
        if (c + 1 < nc) load_block(c + 1, st ^ 1);  // stage st^1 was last read by chunk c-1
      }
      ok = tc::mbar_wait(bar1, par, kWait) && ok;
      tc::fence_after();
      const int t = row;  // token of this W row
#pragma unroll
      for (int piece = 0; piece < 2; ++piece) {  // Vn = U - W S, columns [64 half + 32 piece, +32)
        uint32_t r[32];
        tc::ld32(tP + piece * 32, r);
        tc::wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int col = half * 64 + piece * 32 + q * 8;
          const uint4 uu = *reinterpret_cast<const uint4*>(sb + M::u + M::offu(t, col / 8));
          const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uu);
          uint4 res;
          __nv_bfloat162* r2 = reinterpret_cast<__nv_bfloat162*>(&res);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            r2[e] = __floats2bfloat162_rn(__low2float(u2[e]) - __uint_as_float(r[q * 8 + 2 * e]),
                                          __high2float(u2[e]) - __uint_as_float(r[q * 8 + 2 * e + 1]));
          *reinterpret_cast<uint4*>(smem + M::b2 + M::off16(t, col / 8)) = res;
        }
      }
      tc::fence_async_smem();
      tc::fence_before();
      named_bar(2, 128);  // Vn staged, P's W rows read
      tc::fence_after();
      if (issuer) {  // MMA2: S (+)= K'^T Vn;  MMA3: P += [any; Aqk] Vn (lanes 64-127: O)
#pragma unroll
        for (int s = 0; s < 4; ++s)
          tc::mma_bf16(tmem, tc::smem_desc(sbu + M::a2 + s * 4096, 2048, 128),
                       tc::smem_desc(sbase + M::b2 + s * 4096, 2048, 128), kId2, c > 0 || s > 0);
#pragma unroll
        for (int s = 0; s < 4; ++s)
          tc::mma_bf16(tmem + 128, tc::smem_desc(sbu + M::a3 + s * 256, 128, 1024),
                       tc::smem_desc(sbase + M::b2 + s * 4096, 2048, 128), kId1, true);
        tc::commit(bar2);
      }
    }
    ok = tc::mbar_wait(bar2, par, kWait) && ok;
    tc::fence_after();
    if (!vwarp) {  // O rows (lanes 64..127) -> BF16 stash + row-half sums of squares
      if (c > 0) named_bar(3, 256);  // the norm warps hold chunk c-1's stash
      const int t = row - kC;
      float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int piece = 0; piece < 2; ++piece) {
        uint32_t r[32];
        tc::ld32(tP + piece * 32, r);
        tc::wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            w[e] = bf2_pack(__uint_as_float(r[q * 8 + 2 * e]), __uint_as_float(r[q * 8 + 2 * e + 1]));
            const float2 f = bf2f(w[e]);
            s2 = fma2(f, f, s2);
          }
          *reinterpret_cast<uint4*>(smem + M::ost + M::offu(t, half * 8 + piece * 4 + q)) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      sNss[t * 2 + half] = s2.x + s2.y;
    }
    {  // S: bf16 copy for the next MMA1 (and the final state), then S *= e^{G_last(next chunk)}
      const float f = __expf(gl_next);
      const bool last = c + 1 == nc;
      uint4* dst = reinterpret_cast<uint4*>(a.state + (int64_t(bh) * D + row) * D + half * 64);
#pragma unroll
      for (int piece = 0; piece < 2; ++piece) {
        uint32_t r[32];
        tc::ld32(tS + piece * 32, r);
        tc::wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 res;
          __nv_bfloat162* r2 = reinterpret_cast<__nv_bfloat162*>(&res);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            r2[e] = __floats2bfloat162_rn(__uint_as_float(r[q * 8 + 2 * e]), __uint_as_float(r[q * 8 + 2 * e + 1]));
          *reinterpret_cast<uint4*>(smem + M::b1 + M::off16(row, half * 8 + piece * 4 + q)) = res;
          if (last) dst[piece * 4 + q] = res;
        }
        if (!last) {
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * f);
          tc::st32(tS + piece * 32, r);
        }
      }
      tc::wait_st();
      tc::fence_async_smem();
    }
  }
  ok = __syncthreads_and(ok);  // the last chunk's stash and sums are published
  if (ok && nwarp && nc > 0) norm_chunk(nc - 1, false);
  if (!ok) {  // a wait timed out: report, and give in-flight copies a bounded time to land
    if (tid == 0) atomicOr(a.status, 1u);
    if (issuer)
      for (int st = 0; st < 2; ++st)
        if (ld_issued[st] > 0) tc::mbar_wait(ldbar + st, uint32_t(ld_issued[st] - 1) & 1u, kWait);
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  if (warp == 0) tc::tmem_free(tmem, 256);
}

template <int DK, int DV>
int launch_split(SplitArgs& a, void* ws, int64_t ws_bytes, cudaStream_t s) {
  const int64_t n = int64_t(a.B) * a.HV;
  KB_REQUIRE(ws_bytes >= int64_t(workspace_bytes<DK, DV>(a.B, a.HV, a.L)), KADLLM_EINVAL,
             "gdn prefill: workspace too small");
  a.status = static_cast<uint32_t*>(ws);  // bytes [0, 256): status word; chunk blocks after
  a.blocks = static_cast<unsigned char*>(ws) + 256;
  const bool tc_scan = DK == 128 && DV == 128 && a.ld_out % 8 == 0 && a.ld_proj % 8 == 0 &&
                       (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.state) & 15) == 0 &&
                       (reinterpret_cast<uintptr_t>(a.norm_w) & 15) == 0 &&
                       (reinterpret_cast<uintptr_t>(a.proj) & 15) == 0 && a.rows * a.HV < (1ll << 31);
  KB_REQUIRE(tc_scan || a.cu == nullptr, KADLLM_EUNSUPPORTED,
             "gdn prefill: packed variable-length requests need 128-dim heads and 16-byte aligned rows");
  a.tc_layout = tc_scan ? 1 : 0;
  if (cudaMemsetAsync(a.status, 0, sizeof(uint32_t), s) != cudaSuccess) {
    set_error("gdn prefill: cannot clear the status word");
    return KADLLM_ECUDA;
  }
  if (tc_scan) {
    const size_t smem = PrepTc::bytes;
    if (cudaFuncSetAttribute(gdn_prep_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
      set_error("gdn prefill prep: cannot reserve %zu bytes of shared memory", smem);
      return KADLLM_ECUDA;
    }
    gdn_prep_tc_kernel<<<dim3(a.nc, unsigned(n)), 256, smem, s>>>(a);
    KB_CHECK_LAUNCH("gdn prefill tensor-core prep launch");
  } else {
    const size_t smem = PrepSmem<DK, DV>::bytes;
    auto kern = gdn_prep_kernel<DK, DV>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
      set_error("gdn prefill prep: cannot reserve %zu bytes of shared memory", smem);
      return KADLLM_ECUDA;
    }
    kern<<<dim3(a.nc, unsigned(n)), 256, smem, s>>>(a);
    KB_CHECK_LAUNCH("gdn prefill prep launch");
  }
  if (tc_scan) {
    const size_t smem = TcScan::bytes;
    if (cudaFuncSetAttribute(gdn_scan_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
      set_error("gdn prefill scan: cannot reserve %zu bytes of shared memory", smem);
      return KADLLM_ECUDA;
    }
    gdn_scan_tc_kernel<<<unsigned(n), 384, smem, s>>>(a);
    KB_CHECK_LAUNCH("gdn prefill tensor-core scan launch");
    return KADLLM_OK;
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
  if (batch < 1 || length < 1 || v_heads < 1) return -1;
  if (k_dim == 128 && v_dim == 128) return int64_t(workspace_bytes<128, 128>(batch, v_heads, length));
  if (k_dim == 64 && v_dim == 64) return int64_t(workspace_bytes<64, 64>(batch, v_heads, length));
  if (k_dim == 32 && v_dim == 32) return int64_t(workspace_bytes<32, 32>(batch, v_heads, length));
  return -1;
}

namespace kb {
namespace {
int prefill_split(const void* proj, int64_t ld_proj, const void* conv_weight, void* conv_state, const float* a_log,
                  const float* dt_bias, const float* norm_weight, float norm_eps, void* out, int64_t ld_out,
                  void* state, void* workspace, int64_t workspace_bytes, const int* cu, int64_t rows, int64_t batch,
                  int64_t length, int64_t heads, int64_t v_heads, int64_t k_dim, int64_t v_dim, void* stream) {
  KB_REQUIRE(proj && conv_weight && conv_state && a_log && dt_bias && norm_weight && out && state && workspace,
             KADLLM_EINVAL, "gdn prefill: null pointer");
  KB_REQUIRE(batch >= 1 && length >= 1 && rows >= 1 && heads >= 1 && v_heads >= 1 && v_heads % heads == 0,
             KADLLM_EINVAL, "gdn prefill: bad dimensions");
  KB_REQUIRE(ld_proj % 8 == 0 && ld_out % 2 == 0 && (reinterpret_cast<uintptr_t>(proj) & 15) == 0 &&
                 (reinterpret_cast<uintptr_t>(conv_weight) & 15) == 0 && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0 &&
                 (reinterpret_cast<uintptr_t>(conv_state) & 7) == 0,
             KADLLM_EINVAL, "gdn prefill: projection rows / weights / workspace misaligned");
  const int64_t nc = (length + kC - 1) / kC;
  KB_REQUIRE(nc <= 2147483647 && batch * v_heads <= 65535, KADLLM_EINVAL, "gdn prefill: grid too large");
  SplitArgs a{};
  a.proj = static_cast<const __nv_bfloat16*>(proj); a.ld_proj = ld_proj;
  a.conv_w = static_cast<const __nv_bfloat16*>(conv_weight);
  a.conv_state = static_cast<__nv_bfloat16*>(conv_state);
  a.a_log = a_log; a.dt_bias = dt_bias; a.norm_w = norm_weight; a.eps = norm_eps;
  a.out = static_cast<__nv_bfloat16*>(out); a.ld_out = ld_out;
  a.state = static_cast<__nv_bfloat16*>(state);
  a.cu = cu; a.rows = rows;
  a.B = int(batch); a.L = int(length); a.nc = int(nc); a.H = int(heads); a.HV = int(v_heads);
  a.scale = 1.0f / sqrtf(float(k_dim));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (k_dim == 128 && v_dim == 128) return launch_split<128, 128>(a, workspace, workspace_bytes, s);
  if (k_dim == 64 && v_dim == 64) return launch_split<64, 64>(a, workspace, workspace_bytes, s);
  if (k_dim == 32 && v_dim == 32) return launch_split<32, 32>(a, workspace, workspace_bytes, s);
  set_error("gdn prefill: head dims K=%lld V=%lld must be equal and in {32, 64, 128}", (long long)k_dim,
            (long long)v_dim);
  return KADLLM_EUNSUPPORTED;
}
}  // namespace
}  // namespace kb

extern "C" int kadllm_gdn_prefill_split(const void* proj, int64_t ld_proj, const void* conv_weight, void* conv_state,
                                        const float* a_log, const float* dt_bias, const float* norm_weight,
                                        float norm_eps, void* out, int64_t ld_out, void* state, void* workspace,
                                        int64_t workspace_bytes, int64_t batch, int64_t length, int64_t heads,
                                        int64_t v_heads, int64_t k_dim, int64_t v_dim, void* stream) {
  return kb::prefill_split(proj, ld_proj, conv_weight, conv_state, a_log, dt_bias, norm_weight, norm_eps, out, ld_out,
                           state, workspace, workspace_bytes, nullptr, batch * length, batch, length, heads, v_heads,
                           k_dim, v_dim, stream);
}

extern "C" int kadllm_gdn_prefill_split_varlen(const void* proj, int64_t ld_proj, const void* conv_weight,
                                               void* conv_state, const float* a_log, const float* dt_bias,
                                               const float* norm_weight, float norm_eps, void* out, int64_t ld_out,
                                               void* state, void* workspace, int64_t workspace_bytes,
                                               const int32_t* cu_seqlens, int64_t total_rows, int64_t batch,
                                               int64_t max_length, int64_t heads, int64_t v_heads, int64_t k_dim,
                                               int64_t v_dim, void* stream) {
  KB_REQUIRE(cu_seqlens != nullptr, KADLLM_EINVAL, "gdn prefill: null sequence offsets");
  return kb::prefill_split(proj, ld_proj, conv_weight, conv_state, a_log, dt_bias, norm_weight, norm_eps, out, ld_out,
                           state, workspace, workspace_bytes, cu_seqlens, total_rows, batch, max_length, heads,
                           v_heads, k_dim, v_dim, stream);
}
