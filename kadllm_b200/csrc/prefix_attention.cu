// Shared-prefix attention for beam decode (GQA), plus the per-beam causal suffix.
//
// Semantics: src/kadllm/ops.py:252-341 (prefix_attention): every query row of
// request b attends to the request's prefix keys (non-causal, optional validity
// mask) and to its own beam's suffix keys s <= t; the two partitions are merged
// by log-sum-exp (src/kadllm/ops.py:243-249).  Fully masked / empty prefixes
// contribute nothing.  The FlashAttention path it replaces is
// src/kadllm/kernels/flash_attention.py:11-66.
//
// B200 formulation: all beams of a request share one immutable prefix, so for
// each (request, kv head) the queries of all W beams x T steps x G grouped heads
// form one dense [W*T*G, D] x [D, L] contraction against a single copy of the
// prefix K/V (read once per request from HBM, then from L2).  Each CTA takes 64
// query rows and runs an online-softmax flash loop over 32-key blocks with
// bf16 mma.sync tensor-core tiles and a cp.async double buffer.  The T <= 8
// suffix keys of each beam are merged in the epilogue with fp32 CUDA-core dot
// products.  Optional fused output gate: out = bf16(bf16(o) * bf16(sigmoid(gate)))
// (src/kadllm/adapters/qwen3_5.py:199-201).
#include "common.cuh"

namespace kb {
namespace {

constexpr int kBM = 64;
constexpr int kBN = 32;
constexpr int kThreads = 128;
constexpr int kTMax = 8;
constexpr float kLog2e = 1.4426950408889634f;

struct AttnArgs {
  const __nv_bfloat16* q; int64_t sq_bw, sq_t, sq_h;
  const __nv_bfloat16* pk; int64_t spk_b, spk_l, spk_h;
  const __nv_bfloat16* pv; int64_t spv_b, spv_l, spv_h;
  const __nv_bfloat16* sk; int64_t ssk_bw, ssk_t, ssk_h;
  const __nv_bfloat16* sv; int64_t ssv_bw, ssv_t, ssv_h;
  const uint8_t* mask;  // [B, L] or null
  const __nv_bfloat16* gate; int64_t sg_bw, sg_t, sg_h;  // gate rows / steps / heads, or null
  __nv_bfloat16* out; int64_t so_bw, so_t, so_h;
  int B, W, T, H, HK, G, L;
  float scale_log2;
};

template <int D>
struct AttnSmem {
  static constexpr int kStride = D + 8;
  static constexpr size_t q_elems = size_t(kBM) * kStride;
  static constexpr size_t kv_elems = size_t(kBN) * kStride;
  static constexpr size_t bytes = (q_elems + 4 * kv_elems) * 2 + 2 * kBN * 4 + kBM * kTMax * 4;
};

// CAUSAL = false: beam decode (rows = (beam, t, g), prefix + per-beam suffix).
// CAUSAL = true : prompt prefill (rows = (position, g) of one request, keys are
//                 the request's own positions <= the row's position; q rows are
//                 indexed by token row b * L + position, the suffix is absent).
template <int D, bool CAUSAL>
__global__ void __launch_bounds__(kThreads) prefix_attention_kernel(const AttnArgs a) {
  using S = AttnSmem<D>;
  constexpr int STR = S::kStride;
  constexpr int CH = D / 8;  // 16-byte chunks per row
  extern __shared__ __align__(16) unsigned char smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* sK = sQ + S::q_elems;         // [2][kBN][STR]
  __nv_bfloat16* sV = sK + 2 * S::kv_elems;    // [2][kBN][STR]
  float* sMask = reinterpret_cast<float*>(sV + 2 * S::kv_elems);  // [2][kBN]
  float* sSuf = sMask + 2 * kBN;                                  // [kBM][kTMax]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.y / a.HK, hk = blockIdx.y % a.HK;
  const int TG = a.T * a.G;
  const int R = CAUSAL ? a.L * a.G : a.W * TG;
  const int row0 = blockIdx.x * kBM;

  // ---- Q tile (rows = (beam, t, g) of this request / kv head) -----------------------
  for (int i = tid; i < kBM * CH; i += kThreads) {
    const int r = i / CH, c = i % CH;
    __nv_bfloat16* dst = sQ + r * STR + c * 8;
    const int gr = row0 + r;
    if (gr < R) {
      const __nv_bfloat16* src;
      if constexpr (CAUSAL) {
        const int pos = gr / a.G, g = gr % a.G;
        src = a.q + (int64_t(b) * a.L + pos) * a.sq_bw + int64_t(hk * a.G + g) * a.sq_h + c * 8;
      } else {
        const int beam = gr / TG, rem = gr % TG, t = rem / a.G, g = rem % a.G;
        src = a.q + (int64_t(b) * a.W + beam) * a.sq_bw + int64_t(t) * a.sq_t + int64_t(hk * a.G + g) * a.sq_h + c * 8;
      }
      cp_async16(dst, src);
    } else {
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
  }
  int nkeys = a.L;
  if constexpr (CAUSAL) nkeys = min(a.L, (min(R - 1, row0 + kBM - 1)) / a.G + 1);
  const int nkb = (nkeys + kBN - 1) / kBN;
  auto load_kv = [&](int kb, int buf) {
    for (int i = tid; i < kBN * CH; i += kThreads) {
      const int r = i / CH, c = i % CH;
      const int key = kb * kBN + r;
      __nv_bfloat16* dk = sK + buf * S::kv_elems + r * STR + c * 8;
      __nv_bfloat16* dv = sV + buf * S::kv_elems + r * STR + c * 8;
      if (key < a.L) {
        cp_async16(dk, a.pk + int64_t(b) * a.spk_b + int64_t(key) * a.spk_l + int64_t(hk) * a.spk_h + c * 8);
        cp_async16(dv, a.pv + int64_t(b) * a.spv_b + int64_t(key) * a.spv_l + int64_t(hk) * a.spv_h + c * 8);
      } else {
        *reinterpret_cast<uint4*>(dk) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(dv) = make_uint4(0, 0, 0, 0);
      }
    }
    for (int r = tid; r < kBN; r += kThreads) {
      const int key = kb * kBN + r;
      const bool ok = key < a.L && (a.mask == nullptr || a.mask[int64_t(b) * a.L + key] != 0);
      sMask[buf * kBN + r] = ok ? 0.f : -INFINITY;
    }
  };
  if (nkb > 0) load_kv(0, 0);
  cp_async_commit();

  const int g = lane >> 2, tq = lane & 3;
  // causal: positions of this thread's two rows
  const int cpos0 = (row0 + warp * 16 + g) / a.G, cpos1 = (row0 + warp * 16 + g + 8) / a.G;
  float o[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) {
      load_kv(kb + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16* cK = sK + buf * S::kv_elems;
    const __nv_bfloat16* cV = sV + buf * S::kv_elems;
    // S = Q K^T (16 rows x 32 keys per warp)
    float s[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t af[4];
      ldmatrix_x4(af, sQ + (warp * 16 + (lane & 15)) * STR + kk * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t bk[4];
        ldmatrix_x4(bk, cK + (np * 16 + (lane & 7) + ((lane >> 4) << 3)) * STR + kk * 16 + ((lane >> 3) & 1) * 8);
        const uint32_t b0[2] = {bk[0], bk[1]}, b1[2] = {bk[2], bk[3]};
        mma_bf16_16816(s[2 * np], af, b0);
        mma_bf16_16816(s[2 * np + 1], af, b1);
      }
    }
    // scale, mask, online softmax (log2 domain)
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float ma = sMask[buf * kBN + j * 8 + tq * 2], mb = sMask[buf * kBN + j * 8 + tq * 2 + 1];
      s[j][0] = s[j][0] * a.scale_log2 + ma;
      s[j][1] = s[j][1] * a.scale_log2 + mb;
      s[j][2] = s[j][2] * a.scale_log2 + ma;
      s[j][3] = s[j][3] * a.scale_log2 + mb;
      if constexpr (CAUSAL) {
        const int key = kb * kBN + j * 8 + tq * 2;
        if (key > cpos0) s[j][0] = -INFINITY;
        if (key + 1 > cpos0) s[j][1] = -INFINITY;
        if (key > cpos1) s[j][2] = -INFINITY;
        if (key + 1 > cpos1) s[j][3] = -INFINITY;
      }
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float base0 = mn0 == -INFINITY ? 0.f : mn0, base1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = exp2f(m0 - base0), al1 = exp2f(m1 - base1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      s[j][0] = exp2f(s[j][0] - base0);
      s[j][1] = exp2f(s[j][1] - base0);
      s[j][2] = exp2f(s[j][2] - base1);
      s[j][3] = exp2f(s[j][3] - base1);
      ps0 += s[j][0] + s[j][1];
      ps1 += s[j][2] + s[j][3];
    }
    l0 = l0 * al0 + ps0;
    l1 = l1 * al1 + ps1;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      o[j][0] *= al0; o[j][1] *= al0;
      o[j][2] *= al1; o[j][3] *= al1;
    }
    // O += P V
#pragma unroll
    for (int c = 0; c < kBN / 16; ++c) {
      uint32_t pa[4];
      pa[0] = pack_bf16(s[2 * c][0], s[2 * c][1]);
      pa[1] = pack_bf16(s[2 * c][2], s[2 * c][3]);
      pa[2] = pack_bf16(s[2 * c + 1][0], s[2 * c + 1][1]);
      pa[3] = pack_bf16(s[2 * c + 1][2], s[2 * c + 1][3]);
#pragma unroll
      for (int dn = 0; dn < D / 16; ++dn) {
        uint32_t bv[4];
        ldmatrix_x4_trans(bv, cV + (c * 16 + (lane & 15)) * STR + dn * 16 + (lane >> 4) * 8);
        const uint32_t b0[2] = {bv[0], bv[1]}, b1[2] = {bv[2], bv[3]};
        mma_bf16_16816(o[2 * dn], pa, b0);
        mma_bf16_16816(o[2 * dn + 1], pa, b1);
      }
    }
    __syncthreads();
  }
  if (nkb == 0) cp_async_wait<0>();
  __syncthreads();
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  if constexpr (CAUSAL) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int gr = row0 + warp * 16 + g + half * 8;
      if (gr >= R) continue;
      const int pos = gr / a.G, gg = gr % a.G;
      const float inv = 1.f / (half ? l1 : l0);
      const int64_t trow = int64_t(b) * a.L + pos;
#pragma unroll
      for (int j = 0; j < D / 8; ++j) {
        const int col = j * 8 + tq * 2;
        float v0 = o[j][half * 2] * inv, v1 = o[j][half * 2 + 1] * inv;
        if (a.gate) {
          const __nv_bfloat162 gv =
              *reinterpret_cast<const __nv_bfloat162*>(a.gate + trow * a.sg_bw + int64_t(hk * a.G + gg) * a.sg_h + col);
          v0 = bf16r(v0) * bf16r(sigmoid_f(__low2float(gv)));
          v1 = bf16r(v1) * bf16r(sigmoid_f(__high2float(gv)));
        }
        *reinterpret_cast<__nv_bfloat162*>(a.out + trow * a.so_bw + int64_t(hk * a.G + gg) * a.so_h + col) =
            __floats2bfloat162_rn(v0, v1);
      }
    }
    return;
  }
  // ---- suffix scores: row (beam, t, g) attends to its beam's keys s <= t -----------
  for (int i = 0; i < 16; ++i) {
    const int wr = warp * 16 + i;
    const int gr = row0 + wr;
    if (gr >= R) break;
    const int beam = gr / TG, rem = gr % TG, t = rem / a.G;
    for (int sidx = 0; sidx < a.T; ++sidx) {
      float dot = -INFINITY;
      if (sidx <= t) {
        const __nv_bfloat16* kp = a.sk + (int64_t(b) * a.W + beam) * a.ssk_bw + int64_t(sidx) * a.ssk_t +
                                  int64_t(hk) * a.ssk_h;
        float acc = 0.f;
        for (int d = lane; d < D; d += 32) acc += __bfloat162float(sQ[wr * STR + d]) * __bfloat162float(kp[d]);
        dot = warp_sum(acc) * a.scale_log2;
      }
      if (lane == 0) sSuf[wr * kTMax + sidx] = dot;
    }
  }
  __syncwarp();

  // ---- merge suffix into the running softmax, normalise, gate, store ---------------
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int wr = warp * 16 + g + half * 8;
    const int gr = row0 + wr;
    if (gr >= R) continue;
    const int beam = gr / TG, rem = gr % TG, t = rem / a.G, gg = rem % a.G;
    float m = half ? m1 : m0;
    float l = half ? l1 : l0;
    float mx = m;
    for (int sidx = 0; sidx <= t; ++sidx) mx = fmaxf(mx, sSuf[wr * kTMax + sidx]);
    const float alpha = exp2f(m - mx);  // mx is finite: the suffix always has key t
    l *= alpha;
    float p[kTMax];
#pragma unroll
    for (int sidx = 0; sidx < kTMax; ++sidx) {
      p[sidx] = (sidx <= t && sidx < a.T) ? exp2f(sSuf[wr * kTMax + sidx] - mx) : 0.f;
      l += p[sidx];
    }
    const float inv = 1.f / l;
    const int64_t brow = int64_t(b) * a.W + beam;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      const int col = j * 8 + tq * 2;
      float v0 = o[j][half * 2] * alpha, v1 = o[j][half * 2 + 1] * alpha;
#pragma unroll
      for (int sidx = 0; sidx < kTMax; ++sidx) {
        if (sidx <= t && sidx < a.T) {
          const __nv_bfloat16* vp = a.sv + brow * a.ssv_bw + int64_t(sidx) * a.ssv_t + int64_t(hk) * a.ssv_h + col;
          const __nv_bfloat162 vv = *reinterpret_cast<const __nv_bfloat162*>(vp);
          v0 += p[sidx] * __low2float(vv);
          v1 += p[sidx] * __high2float(vv);
        }
      }
      v0 *= inv;
      v1 *= inv;
      if (a.gate) {
        const __nv_bfloat16* gp = a.gate + brow * a.sg_bw + int64_t(t) * a.sg_t + int64_t(hk * a.G + gg) * a.sg_h + col;
        const __nv_bfloat162 gv = *reinterpret_cast<const __nv_bfloat162*>(gp);
        v0 = bf16r(v0) * bf16r(sigmoid_f(__low2float(gv)));
        v1 = bf16r(v1) * bf16r(sigmoid_f(__high2float(gv)));
      }
      __nv_bfloat16* op = a.out + brow * a.so_bw + int64_t(t) * a.so_t + int64_t(hk * a.G + gg) * a.so_h + col;
      *reinterpret_cast<__nv_bfloat162*>(op) = __floats2bfloat162_rn(v0, v1);
    }
  }
}

template <int D, bool CAUSAL = false>
int launch_attn(const AttnArgs& a, cudaStream_t stream) {
  const size_t smem = AttnSmem<D>::bytes;
  auto kern = prefix_attention_kernel<D, CAUSAL>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
    set_error("attention: cannot reserve %zu bytes of shared memory", smem);
    return KADLLM_ECUDA;
  }
  const int64_t R = CAUSAL ? int64_t(a.L) * a.G : int64_t(a.W) * a.T * a.G;
  dim3 grid(unsigned((R + kBM - 1) / kBM), unsigned(a.B * a.HK));
  kern<<<grid, kThreads, smem, stream>>>(a);
  KB_CHECK_LAUNCH("prefix attention launch");
  return KADLLM_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace kb

extern "C" int kadllm_prefix_attention(
    const void* q, int64_t sq_bw, int64_t sq_t, int64_t sq_h, const void* prefix_k, int64_t spk_b,
    int64_t spk_l, int64_t spk_h, const void* prefix_v, int64_t spv_b, int64_t spv_l, int64_t spv_h,
    const void* suffix_k, int64_t ssk_bw, int64_t ssk_t, int64_t ssk_h, const void* suffix_v,
    int64_t ssv_bw, int64_t ssv_t, int64_t ssv_h, const void* prefix_mask, const void* gate,
    int64_t sg_bw, int64_t sg_t, int64_t sg_h, void* out, int64_t so_bw, int64_t so_t, int64_t so_h, int dtype,
    int64_t batch, int64_t beam_width, int64_t steps, int64_t heads, int64_t kv_heads,
    int64_t prefix_len, int64_t head_dim, float scale, void* stream) {
  using namespace kb;
  KB_REQUIRE(dtype == KADLLM_BF16, KADLLM_EDTYPE, "prefix attention: only bfloat16 is implemented");
  KB_REQUIRE(batch >= 1 && beam_width >= 1 && steps >= 1 && heads >= 1 && kv_heads >= 1 && prefix_len >= 0,
             KADLLM_EINVAL, "prefix attention: empty dimensions");
  KB_REQUIRE(heads % kv_heads == 0, KADLLM_EINVAL, "prefix attention: heads not divisible by kv heads");
  KB_REQUIRE(steps <= kTMax, KADLLM_EUNSUPPORTED, "prefix attention: at most %d suffix steps", kTMax);
  KB_REQUIRE(batch * kv_heads <= 65535, KADLLM_EINVAL, "prefix attention: too many (request, kv head) pairs");
  KB_REQUIRE(q && suffix_k && suffix_v && out && (prefix_len == 0 || (prefix_k && prefix_v)), KADLLM_EINVAL,
             "prefix attention: null pointer");
  // 16-byte cp.async / bf16x2 accesses: rows must start 16-byte aligned
  KB_REQUIRE(aligned16(q) && (prefix_len == 0 || (aligned16(prefix_k) && aligned16(prefix_v))) &&
                 sq_bw % 8 == 0 && sq_t % 8 == 0 && sq_h % 8 == 0 && spk_b % 8 == 0 && spk_l % 8 == 0 &&
                 spk_h % 8 == 0 && spv_b % 8 == 0 && spv_l % 8 == 0 && spv_h % 8 == 0,
             KADLLM_EINVAL, "prefix attention: q / prefix rows must be 16-byte aligned");
  // bf16x2 accesses to suffix K/V, gate and output: even strides, 4-byte aligned bases
  auto even = [](int64_t x) { return (x & 1) == 0; };
  KB_REQUIRE((reinterpret_cast<uintptr_t>(suffix_k) & 3) == 0 && (reinterpret_cast<uintptr_t>(suffix_v) & 3) == 0 &&
                 (reinterpret_cast<uintptr_t>(out) & 3) == 0 && (reinterpret_cast<uintptr_t>(gate) & 3) == 0 &&
                 even(ssk_bw) && even(ssk_t) && even(ssk_h) && even(ssv_bw) && even(ssv_t) && even(ssv_h) &&
                 even(so_bw) && even(so_t) && even(so_h) && even(sg_bw) && even(sg_t) && even(sg_h),
             KADLLM_EINVAL, "prefix attention: suffix / gate / output strides must be even and 4-byte aligned");
  AttnArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q); a.sq_bw = sq_bw; a.sq_t = sq_t; a.sq_h = sq_h;
  a.pk = static_cast<const __nv_bfloat16*>(prefix_k); a.spk_b = spk_b; a.spk_l = spk_l; a.spk_h = spk_h;
  a.pv = static_cast<const __nv_bfloat16*>(prefix_v); a.spv_b = spv_b; a.spv_l = spv_l; a.spv_h = spv_h;
  a.sk = static_cast<const __nv_bfloat16*>(suffix_k); a.ssk_bw = ssk_bw; a.ssk_t = ssk_t; a.ssk_h = ssk_h;
  a.sv = static_cast<const __nv_bfloat16*>(suffix_v); a.ssv_bw = ssv_bw; a.ssv_t = ssv_t; a.ssv_h = ssv_h;
  a.mask = static_cast<const uint8_t*>(prefix_mask);
  a.gate = static_cast<const __nv_bfloat16*>(gate); a.sg_bw = sg_bw; a.sg_t = sg_t; a.sg_h = sg_h;
  a.out = static_cast<__nv_bfloat16*>(out); a.so_bw = so_bw; a.so_t = so_t; a.so_h = so_h;
  a.B = int(batch); a.W = int(beam_width); a.T = int(steps); a.H = int(heads); a.HK = int(kv_heads);
  a.G = int(heads / kv_heads); a.L = int(prefix_len);
  a.scale_log2 = scale * kLog2e;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (head_dim) {
    case 32: return launch_attn<32>(a, s);
    case 64: return launch_attn<64>(a, s);
    case 128: return launch_attn<128>(a, s);
    case 256: return launch_attn<256>(a, s);
    default:
      set_error("prefix attention: head_dim %lld not in {32, 64, 128, 256}", (long long)head_dim);
      return KADLLM_EUNSUPPORTED;
  }
}

extern "C" int kadllm_causal_attention(const void* q, int64_t sq_row, int64_t sq_h, const void* k, int64_t sk_b,
                                       int64_t sk_l, int64_t sk_h, const void* v, int64_t sv_b, int64_t sv_l,
                                       int64_t sv_h, const void* gate, int64_t sg_row, int64_t sg_h, void* out,
                                       int64_t so_row, int64_t so_h, int64_t batch, int64_t length, int64_t heads,
                                       int64_t kv_heads, int64_t head_dim, float scale, void* stream) {
  using namespace kb;
  KB_REQUIRE(q && k && v && out, KADLLM_EINVAL, "causal attention: null pointer");
  KB_REQUIRE(batch >= 1 && length >= 1 && heads >= 1 && kv_heads >= 1 && heads % kv_heads == 0, KADLLM_EINVAL,
             "causal attention: bad dimensions");
  KB_REQUIRE(batch * kv_heads <= 65535, KADLLM_EINVAL, "causal attention: too many (request, kv head) pairs");
  KB_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v) && sq_row % 8 == 0 && sq_h % 8 == 0 && sk_b % 8 == 0 &&
                 sk_l % 8 == 0 && sk_h % 8 == 0 && sv_b % 8 == 0 && sv_l % 8 == 0 && sv_h % 8 == 0,
             KADLLM_EINVAL, "causal attention: rows must be 16-byte aligned");
  KB_REQUIRE((reinterpret_cast<uintptr_t>(out) & 3) == 0 && (reinterpret_cast<uintptr_t>(gate) & 3) == 0 &&
                 so_row % 2 == 0 && so_h % 2 == 0 && sg_row % 2 == 0 && sg_h % 2 == 0,
             KADLLM_EINVAL, "causal attention: gate / output strides must be even");
  AttnArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q); a.sq_bw = sq_row; a.sq_t = 0; a.sq_h = sq_h;
  a.pk = static_cast<const __nv_bfloat16*>(k); a.spk_b = sk_b; a.spk_l = sk_l; a.spk_h = sk_h;
  a.pv = static_cast<const __nv_bfloat16*>(v); a.spv_b = sv_b; a.spv_l = sv_l; a.spv_h = sv_h;
  a.gate = static_cast<const __nv_bfloat16*>(gate); a.sg_bw = sg_row; a.sg_t = 0; a.sg_h = sg_h;
  a.out = static_cast<__nv_bfloat16*>(out); a.so_bw = so_row; a.so_t = 0; a.so_h = so_h;
  a.B = int(batch); a.W = 1; a.T = 1; a.H = int(heads); a.HK = int(kv_heads); a.G = int(heads / kv_heads);
  a.L = int(length);
  a.scale_log2 = scale * kLog2e;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (head_dim) {
    case 32: return launch_attn<32, true>(a, s);
    case 64: return launch_attn<64, true>(a, s);
    case 128: return launch_attn<128, true>(a, s);
    case 256: return launch_attn<256, true>(a, s);
    default:
      set_error("causal attention: head_dim %lld not in {32, 64, 128, 256}", (long long)head_dim);
      return KADLLM_EUNSUPPORTED;
  }
}
