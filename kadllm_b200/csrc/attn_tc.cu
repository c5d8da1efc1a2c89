// Attention over a tiled K/V prefix on the 5th-generation tensor cores
// (head_dim 256): beam decode (shared prefix + per-beam causal suffix) and
// prompt prefill (causal).
//
// Semantics: src/kadllm/ops.py:252-341 (prefix_attention: softmax over the
// request's prefix keys and the beam's own suffix keys s <= t, merged by
// log-sum-exp) and the SDPA call of Qwen3_5Attention on the prompt
// (transformers/models/qwen3_5/modeling_qwen3_5.py:620-692), with the output
// gate out = bf16(bf16(o) * bf16(sigmoid(gate))) (src/kadllm/adapters/
// qwen3_5.py:199-201).
//
// Tiled prefix: for each (request, kv head) the keys (and values) sit in
// blocks of 64 positions x 256 dims, each block a 32 KB core-matrix image
// [8-position group][32 dim chunks][8 positions][16 bytes]: read as a K-major B
// operand (rows = keys) for S = Q K^T and as an MN-major B operand (rows =
// dims) for O += P V, and staged with one bulk copy.  kadllm_kv_tile builds it
// from the [B, HK, L, D] cache, zero-padding the last block.
//
// One CTA = 128 query rows of one (request, kv head), 10 warps.  Query row r
// (TMEM lane r) has two threads, r in warps 0-3 and r + 128 in warps 4-7 (the
// same lane quadrant): they split each block's 64 key columns and the 256
// output columns in halves, exchanging the block maximum through shared memory
// so that both move the softmax reference identically.  Warp 8 issues every
// MMA; warp 9 issues the bulk copies, refilling a K buffer when the S MMA that
// read it completes and a V buffer when its O MMA completes (per-buffer
// barriers), so neither the softmax threads nor the MMA issuer wait behind a
// copy, and the block barrier joins only the row warps and the MMA warp.
// TMEM: S double buffer (2 x 64 columns), O (256 columns).  Per key block j:
// MMA_S(j+1) runs while the row threads turn S(j) into probabilities (exp2
// domain; the reference maximum only moves when a row maximum exceeds it by 8,
// so O is rescaled rarely) and write P (BF16, K-major core tile) to shared
// memory; after the block barrier the issuer starts O += P V(j).  K and V blocks
// are double-buffered.  The epilogue's gate and suffix rows are staged during
// the last key block.  Every mbarrier wait is bounded and reports through a
// status word.
#include "tcgen05.cuh"

namespace kb {
namespace {

constexpr int kD = 256;      // head dim
constexpr int kRows = 128;   // query rows per CTA
constexpr int kBlk = 64;     // keys per block
constexpr int kTile = kBlk * kD * 2;  // bytes of one K or V block (32 KB)
constexpr int kSufMax = 8;
constexpr int kRowThreads = 2 * kRows;  // two threads per query row: key columns / output columns split in halves
constexpr int kThreads = kRowThreads + 64;  // + one warp that issues the MMAs, one that issues the bulk copies
constexpr int kIssuer = kRowThreads;        // the MMA-issuing thread
constexpr int kProducer = kRowThreads + 32; // the copy-issuing thread
constexpr int kBlockSync = kRowThreads + 32;  // threads of the per-block barrier: row warps + MMA warp

struct AttnTcArgs {
  const __nv_bfloat16* q; int64_t sq_row, sq_t, sq_h;  // decode: row = beam row; causal: row = token b*L + pos
  const unsigned char* kt; const unsigned char* vt;     // tiled prefix [B*HK][nblk][kTile]
  int nblk;
  const __nv_bfloat16* sk; int64_t ssk_row, ssk_t, ssk_h;  // decode suffix keys / values
  const __nv_bfloat16* sv; int64_t ssv_row, ssv_t, ssv_h;
  const __nv_bfloat16* gate; int64_t sg_row, sg_t, sg_h;
  __nv_bfloat16* out; int64_t so_row, so_t, so_h;
  uint32_t* status;
  const int* cu;  // varlen prompts: request b's tokens are rows [cu[b], cu[b+1]) (null: b*L .. +L)
  int B, W, T, H, HK, G, L;  // L: the (longest) prefix length
  int t0;                    // decode: first suffix step with query rows (rows for steps t0 .. T-1)
  // decode split over the key blocks (nsplit > 1): CTA z takes blocks [z * bps, (z + 1) * bps) and
  // writes its unnormalised O and (reference maximum, sum) per row; a combine kernel merges the
  // splits with the suffix keys and applies the gate
  int nsplit, bps;
  float* part_o;    // [nsplit][B * HK * R][kD]
  float2* part_ml;  // [nsplit][B * HK * R]
  float scale_log2;
};

struct AttnTcSmem {
  static constexpr size_t q = 0;                                 // [128 rows][256] K-major core tile
  static constexpr size_t k = q + size_t(kRows) * kD * 2;        // K blocks [2]
  static constexpr size_t v = k + 2 * size_t(kTile);             // V blocks [2]
  static constexpr size_t p = v + 2 * size_t(kTile);             // P [128 rows][64 keys] K-major core tile
  static constexpr size_t bm = p + size_t(kRows) * kBlk * 2;     // [2 halves][128 rows] fp32 exchange
  static constexpr size_t bar = bm + size_t(2) * kRows * 4;       // ldK[2], ldV[2], S[2], O, vfree[2]
  static constexpr size_t slot = bar + 9 * 8;
  static constexpr size_t bytes = slot + 8;
  static_assert(bytes <= 232448, "shared memory");
  // 16-byte unit (row r, chunk c) of a core tile whose rows have `chunks` 16-byte chunks
  __device__ static uint32_t off(int r, int c, int chunks) { return (r >> 3) * (chunks * 128) + c * 128 + (r & 7) * 16; }
};

// AND of `v` over the row warps and the MMA warp (named barrier 2)
__device__ __forceinline__ bool block_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.and.pred p, 2, %2, q;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(r)
      : "r"(uint32_t(v)), "n"(kBlockSync)
      : "memory");
  return r != 0;
}

template <bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1) attn_tc_kernel(const AttnTcArgs a) {
  using M = AttnTcSmem;
  constexpr long long kWait = 1ll << 31;
  constexpr uint32_t kIdS = tc::idesc_bf16(kRows, kBlk, 0, 0);  // S = Q K^T: K-major Q and K
  constexpr uint32_t kIdO = tc::idesc_bf16(kRows, kD, 0, 1);    // O += P V: K-major P, MN-major V
  extern __shared__ __align__(16) unsigned char smem[];
  uint64_t* ldK = reinterpret_cast<uint64_t*>(smem + M::bar);  // [2]
  uint64_t* ldV = ldK + 2;                                      // [2]
  uint64_t* barS = ldK + 4;                                     // [2]
  uint64_t* barO = ldK + 6;
  uint64_t* vfree = ldK + 7;                                    // [2]: the O MMA that read V buffer s completed
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + M::slot);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = tid & (kRows - 1), half = (tid / kRows) & 1;  // query row, column half
  const bool rowthr = tid < kRowThreads;                         // warps 0-7 (warps 8, 9 only issue)
  float* sbm = reinterpret_cast<float*>(smem + M::bm);           // partner exchange [half][row]
  const int b = blockIdx.y / a.HK, hk = blockIdx.y % a.HK;
  const int TG = (a.T - a.t0) * a.G;  // query rows per beam
  int64_t seq0 = int64_t(b) * a.L;  // first prompt row of request b
  int Lb = a.L;                      // its prefix length
  if (a.cu) {
    seq0 = a.cu[b];
    Lb = a.cu[b + 1] - a.cu[b];
  }
  const int R = CAUSAL ? Lb * a.G : a.W * TG;
  const int row0 = blockIdx.x * kRows;
  if (row0 >= R) return;  // past this request's rows (varlen): the whole CTA, before any barrier or TMEM
  const int gr = row0 + row;  // this thread's query row (= TMEM lane row)
  const bool rvalid = gr < R;
  int beam = 0, t = 0, g = 0, pos = 0;
  if (CAUSAL) {
    pos = gr / a.G;
    g = gr % a.G;
  } else {
    beam = gr / TG;
    const int rem = gr % TG;
    t = a.t0 + rem / a.G;
    g = rem % a.G;
  }
  const int hq = hk * a.G + g;
  const int64_t qoff = CAUSAL ? (seq0 + pos) * a.sq_row + int64_t(hq) * a.sq_h
                              : (int64_t(b) * a.W + beam) * a.sq_row + int64_t(t) * a.sq_t + int64_t(hq) * a.sq_h;
  int nkeys = Lb;
  if (CAUSAL) nkeys = min(Lb, min(R - 1, row0 + kRows - 1) / a.G + 1);
  const bool split = !CAUSAL && a.nsplit > 1;
  const int jb = split ? int(blockIdx.z) * a.bps : 0;  // this CTA's first key block
  const int nb = split ? max(0, min(a.bps, (nkeys + kBlk - 1) / kBlk - jb)) : (nkeys + kBlk - 1) / kBlk;
  const unsigned char* ktile = a.kt + int64_t(b * a.HK + hk) * a.nblk * kTile;
  const unsigned char* vtile = a.vt + int64_t(b * a.HK + hk) * a.nblk * kTile;
  const uint32_t sbase = smem_u32(smem);

  // ---- prologue: barriers, TMEM, Q tile, first K / V blocks, MMA_S(0) ----------------
  if (tid == 0) {
    for (int i = 0; i < 9; ++i) tc::mbar_init(ldK + i, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 0) tc::tmem_alloc(slot, 512);
  for (int c = half * (kD / 16); rowthr && c < (half + 1) * (kD / 16); ++c) {  // each half: 16 of the row's chunks
    unsigned char* dst = smem + M::q + M::off(row, c, kD / 8);
    if (rvalid) cp_async16(dst, a.q + qoff + c * 8);
    else *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
  }
  cp_async_commit();
  tc::fence_before();
  __syncthreads();  // barriers initialised, TMEM address published
  tc::fence_after();
  const uint32_t tmem = *slot;
  const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;  // TMEM lane quadrant of this warp
  const uint32_t tO = tmem + 128 + lane_off;
  int issued_k[2] = {0, 0}, issued_v[2] = {0, 0};  // loads issued per buffer (issuer thread)
  auto load_k = [&](int j) {
    const int s = j & 1;
    tc::mbar_expect_tx(ldK + s, uint32_t(kTile));
    tc::bulk_g2s(smem + M::k + s * kTile, ktile + int64_t(jb + j) * kTile, uint32_t(kTile), ldK + s);
    ++issued_k[s];
  };
  auto load_v = [&](int j) {
    const int s = j & 1;
    tc::mbar_expect_tx(ldV + s, uint32_t(kTile));
    tc::bulk_g2s(smem + M::v + s * kTile, vtile + int64_t(jb + j) * kTile, uint32_t(kTile), ldV + s);
    ++issued_v[s];
  };
  auto issue_s = [&](int j) {  // S[j & 1] = Q K_j^T
    const int s = j & 1;
#pragma unroll
    for (int kk = 0; kk < kD / 16; ++kk)
      tc::mma_bf16(tmem + s * kBlk, tc::smem_desc(sbase + M::q + kk * 256, 128, 4096),
                   tc::smem_desc(sbase + M::k + s * kTile + kk * 256, 128, 4096), kIdS, kk > 0);
    tc::commit(barS + s);
  };
  auto issue_o = [&](int j) {  // O (+)= P V_j
    const int s = j & 1;
#pragma unroll
    for (int kk = 0; kk < kBlk / 16; ++kk)
      tc::mma_bf16(tmem + 128, tc::smem_desc(sbase + M::p + kk * 256, 128, 1024),
                   tc::smem_desc(sbase + M::v + s * kTile + kk * 8192, 4096, 128), kIdO, j > 0 || kk > 0);
    tc::commit(barO);
    tc::commit(vfree + s);
  };
  if (tid == kProducer && nb > 0) {
    load_k(0);
    load_v(0);
    if (nb > 1) {
      load_k(1);
      load_v(1);
    }
  }
  cp_async_wait<0>();
  tc::fence_async_smem();
  __syncthreads();  // Q tile staged
  bool ok = true;
  if (tid == kIssuer && nb > 0) {
    ok = tc::mbar_wait(ldK, 0, kWait) && ok;
    tc::fence_after();
    issue_s(0);
  }

  // The epilogue's operands are staged by the row threads during the last key block with one
  // batch of cp.async: the gate rows into the K buffers (free once the last S MMA completed;
  // 512-byte rows, chunk c of row r at c ^ (r % 32)), this CTA's beams' suffix keys / values into
  // the V buffer of block nb - 2 (free once its O MMA completed; that of block 1 when nb = 1).
  const int row_hi = min(row0 + kRows, R) - 1;
  const int beam_lo = CAUSAL ? 0 : row0 / TG;
  const int nbeams = CAUSAL ? 0 : row_hi / TG - beam_lo + 1;
  const bool suf_smem = !CAUSAL && int64_t(nbeams) * a.T * kD * 2 * 2 <= int64_t(kTile);
  unsigned char* const ssuf = smem + M::v + (nb >= 2 ? (nb - 2) & 1 : 1) * kTile;
  auto stage_gate = [&]() {  // this thread's half of its own row
    if (!a.gate || !rvalid) return;
    const __nv_bfloat16* src =
        CAUSAL ? a.gate + (seq0 + pos) * a.sg_row + int64_t(hq) * a.sg_h
               : a.gate + (int64_t(b) * a.W + beam) * a.sg_row + int64_t(t) * a.sg_t + int64_t(hq) * a.sg_h;
#pragma unroll 4
    for (int c = half * (kD / 16); c < (half + 1) * (kD / 16); ++c)
      cp_async16(smem + M::k + row * 512 + ((c ^ (row & 31)) * 16), src + c * 8);
  };
  auto stage_suffix = [&]() {
    if (!suf_smem) return;
    for (int i = tid; i < nbeams * a.T * 2 * (kD / 8); i += kRowThreads) {
      const int c = i % (kD / 8), rest = i / (kD / 8), kv = rest & 1, bs = rest >> 1, sidx = bs % a.T, bi = bs / a.T;
      const int64_t br = int64_t(b) * a.W + beam_lo + bi;
      const __nv_bfloat16* src = kv ? a.sv + br * a.ssv_row + int64_t(sidx) * a.ssv_t + int64_t(hk) * a.ssv_h
                                    : a.sk + br * a.ssk_row + int64_t(sidx) * a.ssk_t + int64_t(hk) * a.ssk_h;
      cp_async16(ssuf + ((bi * a.T + sidx) * 2 + kv) * 512 + c * 16, src + c * 8);
    }
  };

  // ---- key blocks ----------------------------------------------------------------------
  const int key_lim = CAUSAL ? pos : Lb - 1;  // last key this row attends to
  float m_ref = -INFINITY, l = 0.f;            // exp2-domain reference maximum, running sum
  if (tid == kProducer) {  // refill each buffer as soon as the MMA that read it has completed
    for (int j = 0; j + 2 < nb; ++j) {
      ok = tc::mbar_wait(barS + (j & 1), uint32_t(j >> 1) & 1u, kWait) && ok;  // K(j) read by MMA_S(j)
      if (!ok) break;
      load_k(j + 2);
      ok = tc::mbar_wait(vfree + (j & 1), uint32_t(j >> 1) & 1u, kWait) && ok;  // V(j) read by MMA_O(j)
      if (!ok) break;
      load_v(j + 2);
    }
  }
  for (int j = 0; warp < 9 && j < nb; ++j) {  // row warps and the MMA warp
    const int sb = j & 1;
    if (tid == kIssuer && j + 1 < nb) {  // MMA_S(j+1) overlaps this block's softmax
      ok = tc::mbar_wait(ldK + ((j + 1) & 1), uint32_t((j + 1) >> 1) & 1u, kWait) && ok;
      tc::fence_after();
      issue_s(j + 1);
    }
    // online softmax over block j: this thread takes key columns [32 half, 32 half + 32)
    float x[32];
    float pm = -INFINITY;
    if (rowthr) {
      ok = tc::mbar_wait(barS + sb, uint32_t(j >> 1) & 1u, kWait) && ok;
      tc::fence_after();
      if (j == nb - 1) {  // every S MMA has completed: the K buffers are free
        if (!split) {
          stage_gate();
          if (nb == 1) stage_suffix();
        }
        cp_async_commit();
      }
      uint32_t r[32];
      tc::ld32(tmem + lane_off + sb * kBlk + half * 32, r);
      tc::wait_ld();
#pragma unroll
      for (int c = 0; c < 32; ++c) x[c] = __uint_as_float(r[c]);
      const int k0 = (jb + j) * kBlk + half * 32;
      if (k0 + 31 > key_lim) {  // partial block: keys past this row's limit drop out
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (k0 + c > key_lim) x[c] = -INFINITY;
      }
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < 32; ++c) m4[c & 3] = fmaxf(m4[c & 3], x[c]);
      pm = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      sbm[half * kRows + row] = pm;
      asm volatile("bar.sync 1, %0;\n" ::"n"(kRowThreads) : "memory");  // the two halves' maxima
      // both halves see the same block maximum, so they move the reference identically
      const float bmax = fmaxf(pm, sbm[(half ^ 1) * kRows + row]) * a.scale_log2;
      float f = 1.f;
      bool resc = false;
      if (bmax > m_ref + 8.f) {  // move the reference (always on the first finite block)
        f = m_ref == -INFINITY ? 0.f : fast_ex2(m_ref - bmax);
        m_ref = bmax;
        l *= f;
        resc = true;
      }
      const float mr = m_ref == -INFINITY ? 0.f : m_ref;  // all scores are -inf while m_ref is
      uint32_t pk[16];
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        const float p0 = fast_ex2(fmaf(x[c], a.scale_log2, -mr));
        const float p1 = fast_ex2(fmaf(x[c + 1], a.scale_log2, -mr));
        s4[(c >> 1) & 3] += p0 + p1;
        pk[c / 2] = bf2_pack(p0, p1);
      }
      l += (s4[0] + s4[1]) + (s4[2] + s4[3]);  // this half's share of the row sum
      if (j > 0) {  // MMA_O(j-1) complete: P is free and O is stable
        ok = tc::mbar_wait(barO, uint32_t(j - 1) & 1u, kWait) && ok;
        tc::fence_after();
        if (j == nb - 1) {  // O(nb-2) has completed: its V buffer is free
          if (!split) stage_suffix();
          cp_async_commit();
        }
        if (resc) {  // this half's 128 output columns
#pragma unroll 1
          for (int piece = half * (kD / 64); piece < (half + 1) * (kD / 64); ++piece) {
            uint32_t o[32];
            tc::ld32(tO + piece * 32, o);
            tc::wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * f);
            tc::st32(tO + piece * 32, o);
          }
          tc::wait_st();
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(smem + M::p + M::off(row, half * 4 + c, kBlk / 8)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
    }
    tc::fence_async_smem();
    tc::fence_before();
    ok = block_and(ok);  // P staged, S(j) and O rows read / rescaled
    if (!ok) break;
    tc::fence_after();
    if (tid == kIssuer) {
      ok = tc::mbar_wait(ldV + sb, uint32_t(j >> 1) & 1u, kWait) && ok;
      issue_o(j);
    }
  }

  // ---- epilogue: merge the beam's suffix (decode), normalise, gate, store --------------
  // every MMA done: K / V / P buffers free.  Only the row warps and the MMA warp wait: they passed the
  // last block barrier after O(nb-2) completed, so the parity names O(nb-1); the copy warp, which
  // writes nothing more, follows through the barrier below.
  if (ok && nb > 0 && warp < 9) {
    ok = tc::mbar_wait(barO, uint32_t(nb - 1) & 1u, kWait);
    tc::fence_after();
  }
  if (rowthr) sbm[half * kRows + row] = l;  // the halves' partial row sums
  cp_async_wait<0>();                       // this thread's staged gate / suffix rows
  __syncthreads();
  if (rowthr) l = sbm[row] + sbm[kRows + row];
  if (split) {  // unnormalised O relative to m_ref, and (m_ref, l): the combine kernel finishes the row
    const int64_t prow = int64_t(blockIdx.z) * (int64_t(a.B) * a.HK * R) + int64_t(blockIdx.y) * R + gr;
    if (rowthr && half == 0 && rvalid) a.part_ml[prow] = make_float2(m_ref, l);
#pragma unroll 1
    for (int piece = half * (kD / 64); rowthr && piece < (half + 1) * (kD / 64); ++piece) {
      uint32_t r[32];
      tc::ld32(tO + piece * 32, r);  // whole warp (aligned)
      tc::wait_ld();
      if (!rvalid) continue;
      float4* dst = reinterpret_cast<float4*>(a.part_o + prow * kD + piece * 32);
#pragma unroll
      for (int q4 = 0; q4 < 8; ++q4)
        dst[q4] = nb > 0 ? make_float4(__uint_as_float(r[4 * q4]), __uint_as_float(r[4 * q4 + 1]),
                                       __uint_as_float(r[4 * q4 + 2]), __uint_as_float(r[4 * q4 + 3]))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  if (!split) {  // merge the suffix, normalise, gate, store (split rows: the combine kernel)
    const int64_t brow = int64_t(b) * a.W + beam;
    auto suf = [&](int sidx, int kv) -> const __nv_bfloat16* {  // this row's suffix key / value s
      if (suf_smem)
        return reinterpret_cast<const __nv_bfloat16*>(ssuf + (((beam - beam_lo) * a.T + sidx) * 2 + kv) * 512);
      return kv ? a.sv + brow * a.ssv_row + int64_t(sidx) * a.ssv_t + int64_t(hk) * a.ssv_h
                : a.sk + brow * a.ssk_row + int64_t(sidx) * a.ssk_t + int64_t(hk) * a.ssk_h;
    };
    float mx = m_ref, alpha = 1.f, ssum = l;
    float psuf[kSufMax];
  #pragma unroll
    for (int sidx = 0; sidx < kSufMax; ++sidx) psuf[sidx] = 0.f;
    const bool lead = rowthr && half == 0;  // computes the row's scalars
    if (lead && !CAUSAL && rvalid) {
      float xs[kSufMax];
  #pragma unroll
      for (int sidx = 0; sidx < kSufMax; ++sidx) {
        xs[sidx] = -INFINITY;
        if (sidx < a.T && sidx <= t) {  // scores against the beam's own keys s <= t
          const __nv_bfloat16* kp = suf(sidx, 0);
          float acc4[4] = {0.f, 0.f, 0.f, 0.f};
  #pragma unroll 8
          for (int c = 0; c < kD / 8; ++c) {
            const uint4 qv = *reinterpret_cast<const uint4*>(smem + M::q + M::off(row, c, kD / 8));
            const uint4 kv = *reinterpret_cast<const uint4*>(kp + c * 8);
            const uint32_t* qw = reinterpret_cast<const uint32_t*>(&qv);
            const uint32_t* kw = reinterpret_cast<const uint32_t*>(&kv);
  #pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 qf = bf2f(qw[e]), kf = bf2f(kw[e]);
              acc4[e] = fmaf(qf.x, kf.x, fmaf(qf.y, kf.y, acc4[e]));
            }
          }
          xs[sidx] = ((acc4[0] + acc4[1]) + (acc4[2] + acc4[3])) * a.scale_log2;
          mx = fmaxf(mx, xs[sidx]);
        }
      }
      alpha = m_ref == -INFINITY ? 0.f : fast_ex2(m_ref - mx);  // mx is finite: key t always exists
      ssum = l * alpha;
  #pragma unroll
      for (int sidx = 0; sidx < kSufMax; ++sidx) {
        psuf[sidx] = xs[sidx] == -INFINITY ? 0.f : fast_ex2(xs[sidx] - mx);
        ssum += psuf[sidx];
      }
    }
    // the row's normaliser, prefix weight and suffix probabilities, shared with the
    // other half's thread of the same row through the (free) P buffer
    float* sc = reinterpret_cast<float*>(smem + M::p) + row * (2 + kSufMax);
    static_assert(size_t(kRows) * (2 + kSufMax) * 4 <= size_t(kRows) * kBlk * 2, "row scalars fit the P buffer");
    if (lead) {
      sc[0] = alpha;
      sc[1] = 1.f / ssum;
  #pragma unroll
      for (int sidx = 0; sidx < kSufMax; ++sidx) sc[2 + sidx] = psuf[sidx];
    }
    __syncthreads();
    alpha = sc[0];
    const float inv = sc[1];
  #pragma unroll
    for (int sidx = 0; sidx < kSufMax; ++sidx) psuf[sidx] = sc[2 + sidx];
    __nv_bfloat16* op = CAUSAL ? a.out + (seq0 + pos) * a.so_row + int64_t(hq) * a.so_h
                               : a.out + brow * a.so_row + int64_t(t) * a.so_t + int64_t(hq) * a.so_h;
  #pragma unroll 1
    for (int piece = half * (kD / 64); rowthr && piece < (half + 1) * (kD / 64); ++piece) {  // this half's columns
      uint32_t r[32];
      tc::ld32(tO + piece * 32, r);  // whole warp (aligned), stores are per row below
      tc::wait_ld();
      if (!rvalid || nb == 0) continue;
      float o[32];
  #pragma unroll
      for (int c = 0; c < 32; ++c) o[c] = __uint_as_float(r[c]) * alpha;
      if (!CAUSAL) {
  #pragma unroll
        for (int sidx = 0; sidx < kSufMax; ++sidx) {
          if (!(sidx < a.T && sidx <= t)) continue;
          const __nv_bfloat16* vp = suf(sidx, 1) + piece * 32;
  #pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const uint4 vv = *reinterpret_cast<const uint4*>(vp + q4 * 8);
            const uint32_t* vw = reinterpret_cast<const uint32_t*>(&vv);
  #pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 vf = bf2f(vw[e]);
              o[q4 * 8 + 2 * e] = fmaf(psuf[sidx], vf.x, o[q4 * 8 + 2 * e]);
              o[q4 * 8 + 2 * e + 1] = fmaf(psuf[sidx], vf.y, o[q4 * 8 + 2 * e + 1]);
            }
          }
        }
      }
  #pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint4 res;
        uint32_t* rw = reinterpret_cast<uint32_t*>(&res);
        uint4 gv = make_uint4(0u, 0u, 0u, 0u);
        const int c = piece * 4 + q4;
        if (a.gate) gv = *reinterpret_cast<const uint4*>(smem + M::k + row * 512 + ((c ^ (row & 31)) * 16));
        const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gv);
  #pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v0 = o[q4 * 8 + 2 * e] * inv, v1 = o[q4 * 8 + 2 * e + 1] * inv;
          if (a.gate) {  // bf16(o) * bf16(sigmoid(gate)), each pair rounded by one packed conversion
            const float2 gf = bf2f(gw[e]);
            const float2 vr = bf2f(bf2_pack(v0, v1));
            const float2 sr = bf2f(bf2_pack(fast_rcp(1.f + fast_ex2(-1.4426950408889634f * gf.x)),
                                            fast_rcp(1.f + fast_ex2(-1.4426950408889634f * gf.y))));
            v0 = vr.x * sr.x;
            v1 = vr.y * sr.y;
          }
          rw[e] = bf2_pack(v0, v1);
        }
        *reinterpret_cast<uint4*>(op + piece * 32 + q4 * 8) = res;
      }
    }
  }
  if (!ok && (tid == 0 || tid == kIssuer || tid == kProducer)) atomicOr(a.status, 1u);  // a wait timed out
  if (tid == kProducer) {  // every copy has landed (normally consumed already; bounded after a timeout)
    for (int s = 0; s < 2; ++s) {
      if (issued_k[s] > 0) tc::mbar_wait(ldK + s, uint32_t(issued_k[s] - 1) & 1u, kWait);
      if (issued_v[s] > 0) tc::mbar_wait(ldV + s, uint32_t(issued_v[s] - 1) & 1u, kWait);
    }
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  if (warp == 0) tc::tmem_free(tmem, 512);
}

// [S][HK][L][D] (strides in elements: seq, pos, head) -> tiles [S*HK][nblk][kTile], zero past L.
// Thread i writes 16-byte unit i of the destination (consecutive threads, consecutive bytes).
__global__ void __launch_bounds__(256) kv_tile_kernel(const __nv_bfloat16* src, int64_t s_seq, int64_t s_pos,
                                                      int64_t s_h, int HK, int L, int nblk, unsigned char* dst,
                                                      int64_t units, const int* cu) {
  const int64_t i = int64_t(blockIdx.x) * 256 + threadIdx.x;
  if (i >= units) return;
  constexpr int per_blk = kTile / 16;  // 2048 units: [8 key groups][32 dim chunks][8 keys]
  const int64_t blk = i / per_blk;
  const int u = int(i % per_blk);
  const int kg = u >> 8, dc = (u >> 3) & 31, k8 = u & 7;
  const int64_t sh = blk / nblk;
  const int kb = int(blk % nblk);
  const int64_t s = sh / HK;
  const int h = int(sh % HK);
  const int p = kb * kBlk + kg * 8 + k8;
  int64_t base = s * s_seq;  // varlen (cu): sequence s is positions [cu[s], cu[s+1]) of one packed run
  int len = L;
  if (cu) {
    base = int64_t(cu[s]) * s_pos;
    len = cu[s + 1] - cu[s];
  }
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (p < len) v = *reinterpret_cast<const uint4*>(src + base + int64_t(p) * s_pos + int64_t(h) * s_h + dc * 8);
  reinterpret_cast<uint4*>(dst)[i] = v;
}

template <bool CAUSAL>
int launch_attn_tc(const AttnTcArgs& a, cudaStream_t stream) {
  auto kern = attn_tc_kernel<CAUSAL>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(AttnTcSmem::bytes)) != cudaSuccess) {
    set_error("tiled attention: cannot reserve %zu bytes of shared memory", AttnTcSmem::bytes);
    return KADLLM_ECUDA;
  }
  const int64_t R = CAUSAL ? int64_t(a.L) * a.G : int64_t(a.W) * (a.T - a.t0) * a.G;
  dim3 grid(unsigned((R + kRows - 1) / kRows), unsigned(a.B * a.HK), unsigned(CAUSAL ? 1 : max(a.nsplit, 1)));
  kern<<<grid, kThreads, AttnTcSmem::bytes, stream>>>(a);
  KB_CHECK_LAUNCH("tiled attention launch");
  return KADLLM_OK;
}

// Split decode: one warp per query row merges the splits' (O, m, l), the row's suffix keys
// s <= t (scores q.k_s from the row's q, in the kernel's exp2 domain) and values, then
// normalises and applies the gate like the fused epilogue.  Lane i holds dims 8i .. 8i + 7.
__global__ void __launch_bounds__(128) attn_split_combine_kernel(const AttnTcArgs a) {
  const int TG = (a.T - a.t0) * a.G;
  const int64_t R = int64_t(a.W) * TG;
  const int64_t rows = int64_t(a.B) * a.HK * R;
  const int64_t id = int64_t(blockIdx.x) * 4 + (threadIdx.x >> 5);
  if (id >= rows) return;  // whole warp
  const int lane = threadIdx.x & 31;
  const int bh = int(id / R), gr = int(id % R);
  const int b = bh / a.HK, hk = bh % a.HK;
  const int beam = gr / TG, rem = gr % TG, t = a.t0 + rem / a.G, g = rem % a.G, hq = hk * a.G + g;
  const int64_t brow = int64_t(b) * a.W + beam;
  // every load up front (the first kPre splits' partials, q, the suffix keys and values,
  // the gate), then the merge in the order of the fused epilogue
  constexpr int kPre = 4;
  float2 mlp[kPre];
  float4 up[kPre][2];
#pragma unroll
  for (int sp = 0; sp < kPre; ++sp) {
    mlp[sp] = make_float2(-INFINITY, 0.f);
    up[sp][0] = up[sp][1] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (sp < a.nsplit) {
      mlp[sp] = a.part_ml[int64_t(sp) * rows + id];
      const float4* src = reinterpret_cast<const float4*>(a.part_o + (int64_t(sp) * rows + id) * kD + lane * 8);
      up[sp][0] = src[0];
      up[sp][1] = src[1];
    }
  }
  const uint4 qv = *reinterpret_cast<const uint4*>(a.q + brow * a.sq_row + int64_t(t) * a.sq_t + int64_t(hq) * a.sq_h +
                                                   lane * 8);
  constexpr int kSufPre = 4;  // suffix keys / values loaded up front; later ones in the loops below
  uint4 kv[kSufPre], vv[kSufPre];
#pragma unroll
  for (int sidx = 0; sidx < kSufPre; ++sidx) {
    kv[sidx] = vv[sidx] = make_uint4(0u, 0u, 0u, 0u);
    if (sidx < a.T && sidx <= t) {
      kv[sidx] = *reinterpret_cast<const uint4*>(a.sk + brow * a.ssk_row + int64_t(sidx) * a.ssk_t +
                                                 int64_t(hk) * a.ssk_h + lane * 8);
      vv[sidx] = *reinterpret_cast<const uint4*>(a.sv + brow * a.ssv_row + int64_t(sidx) * a.ssv_t +
                                                 int64_t(hk) * a.ssv_h + lane * 8);
    }
  }
  uint4 gv = make_uint4(0u, 0u, 0u, 0u);
  if (a.gate)
    gv = *reinterpret_cast<const uint4*>(a.gate + brow * a.sg_row + int64_t(t) * a.sg_t + int64_t(hq) * a.sg_h +
                                         lane * 8);
  float M = -INFINITY;
#pragma unroll
  for (int sp = 0; sp < kPre; ++sp) M = fmaxf(M, mlp[sp].x);
  for (int sp = kPre; sp < a.nsplit; ++sp) M = fmaxf(M, a.part_ml[int64_t(sp) * rows + id].x);
  // suffix scores
  const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
  float xs[kSufMax];
#pragma unroll
  for (int sidx = 0; sidx < kSufMax; ++sidx) {
    xs[sidx] = -INFINITY;
    if (sidx < a.T && sidx <= t) {
      const uint4 k4 = sidx < kSufPre ? kv[sidx < kSufPre ? sidx : 0]
                                      : *reinterpret_cast<const uint4*>(a.sk + brow * a.ssk_row + int64_t(sidx) * a.ssk_t +
                                                                        int64_t(hk) * a.ssk_h + lane * 8);
      const uint32_t kw[4] = {k4.x, k4.y, k4.z, k4.w};
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 qf = bf2f(qw[e]), kf = bf2f(kw[e]);
        acc = fmaf(qf.x, kf.x, fmaf(qf.y, kf.y, acc));
      }
      xs[sidx] = warp_sum(acc) * a.scale_log2;
      M = fmaxf(M, xs[sidx]);
    }
  }
  float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float L = 0.f;
  auto add_split = [&](float2 ml, float4 u0, float4 u1) {
    if (!(ml.x > -INFINITY)) return;
    const float f = fast_ex2(ml.x - M);
    L = fmaf(ml.y, f, L);
    o[0] = fmaf(u0.x, f, o[0]); o[1] = fmaf(u0.y, f, o[1]); o[2] = fmaf(u0.z, f, o[2]); o[3] = fmaf(u0.w, f, o[3]);
    o[4] = fmaf(u1.x, f, o[4]); o[5] = fmaf(u1.y, f, o[5]); o[6] = fmaf(u1.z, f, o[6]); o[7] = fmaf(u1.w, f, o[7]);
  };
#pragma unroll
  for (int sp = 0; sp < kPre; ++sp) add_split(mlp[sp], up[sp][0], up[sp][1]);
  for (int sp = kPre; sp < a.nsplit; ++sp) {
    const float4* src = reinterpret_cast<const float4*>(a.part_o + (int64_t(sp) * rows + id) * kD + lane * 8);
    add_split(a.part_ml[int64_t(sp) * rows + id], src[0], src[1]);
  }
#pragma unroll
  for (int sidx = 0; sidx < kSufMax; ++sidx) {
    if (!(xs[sidx] > -INFINITY)) continue;
    const float p = fast_ex2(xs[sidx] - M);
    L += p;
    const uint4 v4 = sidx < kSufPre ? vv[sidx < kSufPre ? sidx : 0]
                                    : *reinterpret_cast<const uint4*>(a.sv + brow * a.ssv_row + int64_t(sidx) * a.ssv_t +
                                                                      int64_t(hk) * a.ssv_h + lane * 8);
    const uint32_t vw[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 vf = bf2f(vw[e]);
      o[2 * e] = fmaf(p, vf.x, o[2 * e]);
      o[2 * e + 1] = fmaf(p, vf.y, o[2 * e + 1]);
    }
  }
  const float inv = 1.f / L;
  const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
  uint32_t res[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float v0 = o[2 * e] * inv, v1 = o[2 * e + 1] * inv;
    if (a.gate) {  // bf16(o) * bf16(sigmoid(gate)), as the fused epilogue
      const float2 gf = bf2f(gw[e]);
      const float2 vr = bf2f(bf2_pack(v0, v1));
      const float2 sr = bf2f(bf2_pack(fast_rcp(1.f + fast_ex2(-1.4426950408889634f * gf.x)),
                                      fast_rcp(1.f + fast_ex2(-1.4426950408889634f * gf.y))));
      v0 = vr.x * sr.x;
      v1 = vr.y * sr.y;
    }
    res[e] = bf2_pack(v0, v1);
  }
  *reinterpret_cast<uint4*>(a.out + brow * a.so_row + int64_t(t) * a.so_t + int64_t(hq) * a.so_h + lane * 8) =
      make_uint4(res[0], res[1], res[2], res[3]);
}

}  // namespace
}  // namespace kb

using namespace kb;

extern "C" int64_t kadllm_kv_tile_bytes(int64_t seqs, int64_t kv_heads, int64_t length, int64_t head_dim) {
  if (seqs < 1 || kv_heads < 1 || length < 1 || head_dim != kD) return -1;
  return seqs * kv_heads * ((length + kBlk - 1) / kBlk) * int64_t(kTile);
}

namespace kb {
namespace {
int kv_tile(const void* src, int64_t s_seq, int64_t s_pos, int64_t s_head, const int* cu, int64_t seqs,
            int64_t kv_heads, int64_t length, int64_t head_dim, void* tiles, int64_t tile_bytes, void* stream) {
  KB_REQUIRE(src && tiles, KADLLM_EINVAL, "kv_tile: null pointer");
  KB_REQUIRE(head_dim == kD && seqs >= 1 && kv_heads >= 1 && length >= 1, KADLLM_EUNSUPPORTED,
             "kv_tile: head_dim must be %d", kD);
  KB_REQUIRE(s_seq % 8 == 0 && s_pos % 8 == 0 && s_head % 8 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0 &&
                 (reinterpret_cast<uintptr_t>(tiles) & 15) == 0,
             KADLLM_EINVAL, "kv_tile: source rows must be 16-byte aligned");
  const int64_t nblk = (length + kBlk - 1) / kBlk;
  const int64_t bytes = seqs * kv_heads * nblk * kTile;
  KB_REQUIRE(tile_bytes >= bytes, KADLLM_EINVAL, "kv_tile: tile buffer too small (%lld < %lld)", (long long)tile_bytes,
             (long long)bytes);
  const int64_t units = bytes / 16;
  kv_tile_kernel<<<unsigned((units + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(src), s_seq, s_pos, s_head, int(kv_heads), int(length), int(nblk),
      static_cast<unsigned char*>(tiles), units, cu);
  KB_CHECK_LAUNCH("kv_tile launch");
  return KADLLM_OK;
}
}  // namespace
}  // namespace kb

extern "C" int kadllm_kv_tile(const void* src, int64_t s_seq, int64_t s_pos, int64_t s_head, int64_t seqs,
                              int64_t kv_heads, int64_t length, int64_t head_dim, void* tiles, int64_t tile_bytes,
                              void* stream) {
  return kb::kv_tile(src, s_seq, s_pos, s_head, nullptr, seqs, kv_heads, length, head_dim, tiles, tile_bytes, stream);
}

extern "C" int kadllm_kv_tile_varlen(const void* src, int64_t s_pos, int64_t s_head, const int32_t* cu_seqlens,
                                     int64_t seqs, int64_t kv_heads, int64_t max_length, int64_t head_dim, void* tiles,
                                     int64_t tile_bytes, void* stream) {
  KB_REQUIRE(cu_seqlens != nullptr, KADLLM_EINVAL, "kv_tile: null sequence offsets");
  return kb::kv_tile(src, 0, s_pos, s_head, cu_seqlens, seqs, kv_heads, max_length, head_dim, tiles, tile_bytes,
                     stream);
}

namespace kb {
namespace {
int attention_tiled(const void* q, int64_t sq_row, int64_t sq_t, int64_t sq_h, const void* k_tiles,
                    const void* v_tiles, int64_t blocks_per_head, const void* suffix_k, int64_t ssk_row,
                    int64_t ssk_t, int64_t ssk_h, const void* suffix_v, int64_t ssv_row, int64_t ssv_t, int64_t ssv_h,
                    const void* gate, int64_t sg_row, int64_t sg_t, int64_t sg_h, void* out, int64_t so_row,
                    int64_t so_t, int64_t so_h, uint32_t* status, const int* cu, int64_t batch, int64_t beam_width,
                    int64_t steps, int64_t first_step, int64_t q_heads, int64_t kv_heads, int64_t prefix_len,
                    int64_t head_dim, float scale, int causal, void* stream) {
  KB_REQUIRE(q && k_tiles && v_tiles && out && status, KADLLM_EINVAL, "tiled attention: null pointer");
  KB_REQUIRE(first_step >= 0 && (causal ? first_step == 0 : first_step < steps), KADLLM_EINVAL,
             "tiled attention: first_step must lie in [0, steps) (0 for prefill)");
  KB_REQUIRE(head_dim == kD, KADLLM_EUNSUPPORTED, "tiled attention: head_dim must be %d", kD);
  KB_REQUIRE(batch >= 1 && q_heads >= 1 && kv_heads >= 1 && q_heads % kv_heads == 0 && prefix_len >= 1 &&
                 blocks_per_head * kBlk >= prefix_len,
             KADLLM_EINVAL, "tiled attention: bad dimensions");
  if (!causal)
    KB_REQUIRE(suffix_k && suffix_v && beam_width >= 1 && steps >= 1 && steps <= kSufMax, KADLLM_EINVAL,
               "tiled attention: decode needs suffix keys / values and 1 <= steps <= %d", kSufMax);
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  KB_REQUIRE(al16(q) && al16(k_tiles) && al16(v_tiles) && al16(out) && (!suffix_k || al16(suffix_k)) &&
                 (!suffix_v || al16(suffix_v)) && (!gate || al16(gate)) && sq_row % 8 == 0 && sq_t % 8 == 0 &&
                 sq_h % 8 == 0 && so_row % 8 == 0 && so_t % 8 == 0 && so_h % 8 == 0 && ssk_row % 8 == 0 &&
                 ssk_t % 8 == 0 && ssk_h % 8 == 0 && ssv_row % 8 == 0 && ssv_t % 8 == 0 && ssv_h % 8 == 0 &&
                 sg_row % 8 == 0 && sg_t % 8 == 0 && sg_h % 8 == 0,
             KADLLM_EINVAL, "tiled attention: operands and strides must be 16-byte aligned");
  const int64_t R = causal ? prefix_len * (q_heads / kv_heads) : beam_width * (steps - first_step) * (q_heads / kv_heads);
  KB_REQUIRE(R < (int64_t(1) << 30) && batch * kv_heads <= 65535, KADLLM_EINVAL, "tiled attention: too many rows");
  AttnTcArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q); a.sq_row = sq_row; a.sq_t = sq_t; a.sq_h = sq_h;
  a.kt = static_cast<const unsigned char*>(k_tiles); a.vt = static_cast<const unsigned char*>(v_tiles);
  a.nblk = int(blocks_per_head);
  a.sk = static_cast<const __nv_bfloat16*>(suffix_k); a.ssk_row = ssk_row; a.ssk_t = ssk_t; a.ssk_h = ssk_h;
  a.sv = static_cast<const __nv_bfloat16*>(suffix_v); a.ssv_row = ssv_row; a.ssv_t = ssv_t; a.ssv_h = ssv_h;
  a.gate = static_cast<const __nv_bfloat16*>(gate); a.sg_row = sg_row; a.sg_t = sg_t; a.sg_h = sg_h;
  a.out = static_cast<__nv_bfloat16*>(out); a.so_row = so_row; a.so_t = so_t; a.so_h = so_h;
  a.status = status;
  a.cu = cu;
  a.B = int(batch); a.W = int(causal ? 1 : beam_width); a.T = int(causal ? 1 : steps); a.H = int(q_heads);
  a.HK = int(kv_heads); a.G = int(q_heads / kv_heads); a.L = int(prefix_len); a.t0 = int(first_step);
  a.scale_log2 = (scale > 0.f ? scale : 1.0f / sqrtf(float(head_dim))) * 1.4426950408889634f;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return causal ? launch_attn_tc<true>(a, s) : launch_attn_tc<false>(a, s);
}
}  // namespace
}  // namespace kb

extern "C" int kadllm_attention_tiled(const void* q, int64_t sq_row, int64_t sq_t, int64_t sq_h, const void* k_tiles,
                                      const void* v_tiles, int64_t blocks_per_head, const void* suffix_k,
                                      int64_t ssk_row, int64_t ssk_t, int64_t ssk_h, const void* suffix_v,
                                      int64_t ssv_row, int64_t ssv_t, int64_t ssv_h, const void* gate, int64_t sg_row,
                                      int64_t sg_t, int64_t sg_h, void* out, int64_t so_row, int64_t so_t,
                                      int64_t so_h, uint32_t* status, int64_t batch, int64_t beam_width,
                                      int64_t steps, int64_t first_step, int64_t q_heads, int64_t kv_heads,
                                      int64_t prefix_len, int64_t head_dim, float scale, int causal, void* stream) {
  return kb::attention_tiled(q, sq_row, sq_t, sq_h, k_tiles, v_tiles, blocks_per_head, suffix_k, ssk_row, ssk_t,
                             ssk_h, suffix_v, ssv_row, ssv_t, ssv_h, gate, sg_row, sg_t, sg_h, out, so_row, so_t,
                             so_h, status, nullptr, batch, beam_width, steps, first_step, q_heads, kv_heads,
                             prefix_len, head_dim, scale, causal, stream);
}

extern "C" int kadllm_attention_tiled_varlen(
    const void* q, int64_t sq_row, int64_t sq_t, int64_t sq_h, const void* k_tiles, const void* v_tiles,
    int64_t blocks_per_head, const void* suffix_k, int64_t ssk_row, int64_t ssk_t, int64_t ssk_h,
    const void* suffix_v, int64_t ssv_row, int64_t ssv_t, int64_t ssv_h, const void* gate, int64_t sg_row,
    int64_t sg_t, int64_t sg_h, void* out, int64_t so_row, int64_t so_t, int64_t so_h, uint32_t* status,
    const int32_t* cu_seqlens, int64_t batch, int64_t beam_width, int64_t steps, int64_t first_step,
    int64_t q_heads, int64_t kv_heads, int64_t max_prefix_len, int64_t head_dim, float scale, int causal,
    void* stream) {
  KB_REQUIRE(cu_seqlens != nullptr, KADLLM_EINVAL, "tiled attention: null sequence offsets");
  return kb::attention_tiled(q, sq_row, sq_t, sq_h, k_tiles, v_tiles, blocks_per_head, suffix_k, ssk_row, ssk_t,
                             ssk_h, suffix_v, ssv_row, ssv_t, ssv_h, gate, sg_row, sg_t, sg_h, out, so_row, so_t,
                             so_h, status, cu_seqlens, batch, beam_width, steps, first_step, q_heads, kv_heads,
                             max_prefix_len, head_dim, scale, causal, stream);
}

namespace kb {
namespace {
// Bytes of the split partials for a decode launch (0 when no split is taken).
int64_t split_bytes(int64_t batch, int64_t beam_width, int64_t steps, int64_t first_step, int64_t q_heads,
                    int64_t splits) {
  if (splits <= 1) return 0;
  const int64_t rows = batch * beam_width * (steps - first_step) * q_heads;
  return ((splits * rows * 8 + 255) & ~int64_t(255)) + splits * rows * int64_t(kD) * 4;  // (m, l), then O
}
}  // namespace
}  // namespace kb

extern "C" int64_t kadllm_attention_split_workspace(int64_t batch, int64_t beam_width, int64_t steps,
                                                    int64_t first_step, int64_t q_heads, int64_t splits) {
  if (batch < 1 || beam_width < 1 || steps < 1 || first_step < 0 || first_step >= steps || q_heads < 1) return -1;
  return kb::split_bytes(batch, beam_width, steps, first_step, q_heads, splits);
}

extern "C" int kadllm_attention_tiled_split(const void* q, int64_t sq_row, int64_t sq_t, int64_t sq_h,
                                            const void* k_tiles, const void* v_tiles, int64_t blocks_per_head,
                                            const void* suffix_k, int64_t ssk_row, int64_t ssk_t, int64_t ssk_h,
                                            const void* suffix_v, int64_t ssv_row, int64_t ssv_t, int64_t ssv_h,
                                            const void* gate, int64_t sg_row, int64_t sg_t, int64_t sg_h, void* out,
                                            int64_t so_row, int64_t so_t, int64_t so_h, uint32_t* status,
                                            int64_t batch, int64_t beam_width, int64_t steps, int64_t first_step,
                                            int64_t q_heads, int64_t kv_heads, int64_t prefix_len, int64_t head_dim,
                                            float scale, int64_t splits, void* workspace, int64_t workspace_bytes,
                                            void* stream) {
  using namespace kb;
  const int64_t nblk_keys = (prefix_len + kBlk - 1) / kBlk;
  if (splits > nblk_keys) splits = nblk_keys;
  if (splits <= 1)
    return attention_tiled(q, sq_row, sq_t, sq_h, k_tiles, v_tiles, blocks_per_head, suffix_k, ssk_row, ssk_t, ssk_h,
                           suffix_v, ssv_row, ssv_t, ssv_h, gate, sg_row, sg_t, sg_h, out, so_row, so_t, so_h, status,
                           nullptr, batch, beam_width, steps, first_step, q_heads, kv_heads, prefix_len, head_dim,
                           scale, 0, stream);
  KB_REQUIRE(splits <= 64, KADLLM_EINVAL, "tiled attention: at most 64 splits");
  const int64_t bps = (nblk_keys + splits - 1) / splits;
  splits = (nblk_keys + bps - 1) / bps;  // every split holds at least one key block
  const int64_t need = split_bytes(batch, beam_width, steps, first_step, q_heads, splits);
  KB_REQUIRE(workspace && workspace_bytes >= need && (reinterpret_cast<uintptr_t>(workspace) & 15) == 0,
             KADLLM_EINVAL, "tiled attention: split workspace too small (%lld bytes needed)", (long long)need);
  KB_REQUIRE(q && k_tiles && v_tiles && out && status && suffix_k && suffix_v, KADLLM_EINVAL,
             "tiled attention: null pointer");
  KB_REQUIRE(head_dim == kD, KADLLM_EUNSUPPORTED, "tiled attention: head_dim must be %d", kD);
  KB_REQUIRE(batch >= 1 && q_heads >= 1 && kv_heads >= 1 && q_heads % kv_heads == 0 && prefix_len >= 1 &&
                 blocks_per_head * kBlk >= prefix_len && beam_width >= 1 && steps >= 1 && steps <= kSufMax &&
                 first_step >= 0 && first_step < steps,
             KADLLM_EINVAL, "tiled attention: bad dimensions");
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  KB_REQUIRE(al16(q) && al16(k_tiles) && al16(v_tiles) && al16(out) && al16(suffix_k) && al16(suffix_v) &&
                 (!gate || al16(gate)) && sq_row % 8 == 0 && sq_t % 8 == 0 && sq_h % 8 == 0 && so_row % 8 == 0 &&
                 so_t % 8 == 0 && so_h % 8 == 0 && ssk_row % 8 == 0 && ssk_t % 8 == 0 && ssk_h % 8 == 0 &&
                 ssv_row % 8 == 0 && ssv_t % 8 == 0 && ssv_h % 8 == 0 && sg_row % 8 == 0 && sg_t % 8 == 0 &&
                 sg_h % 8 == 0,
             KADLLM_EINVAL, "tiled attention: operands and strides must be 16-byte aligned");
  const int64_t R = beam_width * (steps - first_step) * (q_heads / kv_heads);
  KB_REQUIRE(R < (int64_t(1) << 30) && batch * kv_heads <= 65535, KADLLM_EINVAL, "tiled attention: too many rows");
  AttnTcArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q); a.sq_row = sq_row; a.sq_t = sq_t; a.sq_h = sq_h;
  a.kt = static_cast<const unsigned char*>(k_tiles); a.vt = static_cast<const unsigned char*>(v_tiles);
  a.nblk = int(blocks_per_head);
  a.sk = static_cast<const __nv_bfloat16*>(suffix_k); a.ssk_row = ssk_row; a.ssk_t = ssk_t; a.ssk_h = ssk_h;
  a.sv = static_cast<const __nv_bfloat16*>(suffix_v); a.ssv_row = ssv_row; a.ssv_t = ssv_t; a.ssv_h = ssv_h;
  a.gate = static_cast<const __nv_bfloat16*>(gate); a.sg_row = sg_row; a.sg_t = sg_t; a.sg_h = sg_h;
  a.out = static_cast<__nv_bfloat16*>(out); a.so_row = so_row; a.so_t = so_t; a.so_h = so_h;
  a.status = status;
  a.B = int(batch); a.W = int(beam_width); a.T = int(steps); a.H = int(q_heads);
  a.HK = int(kv_heads); a.G = int(q_heads / kv_heads); a.L = int(prefix_len); a.t0 = int(first_step);
  a.scale_log2 = (scale > 0.f ? scale : 1.0f / sqrtf(float(head_dim))) * 1.4426950408889634f;
  a.nsplit = int(splits);
  a.bps = int(bps);
  const int64_t rows = batch * kv_heads * R;
  a.part_ml = static_cast<float2*>(workspace);
  a.part_o = reinterpret_cast<float*>(static_cast<char*>(workspace) + ((splits * rows * 8 + 255) & ~int64_t(255)));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int rc = launch_attn_tc<false>(a, s)) return rc;
  attn_split_combine_kernel<<<unsigned((rows + 3) / 4), 128, 0, s>>>(a);
  KB_CHECK_LAUNCH("tiled attention split combine launch");
  return KADLLM_OK;
}
