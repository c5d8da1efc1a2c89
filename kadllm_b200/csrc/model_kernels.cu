// Row-wise kernels of the Qwen3.5 hybrid decoder (BF16), each HBM-bound.
//
//   embed_rmsnorm   x = embed[ids]; normed = RMSNorm(x)          (TF:1227-1290 + TF:711-728)
//   add_rmsnorm     x = bf16(x + delta); normed = RMSNorm(x)    (residual + next norm, TF:744-783)
//   silu_mul        act = bf16(bf16(silu(gate)) * up)            (Qwen3_5MLP, TF:695-708)
//   qk_norm_rope    per-head RMSNorm (1+w) of q and k, partial RoPE on the first
//                   rotary_dim dims, scatter q / k / v to their destinations
//                   (Qwen3_5Attention q/k path, TF:661-676; rotary TF:566-595)
// TF: transformers/models/qwen3_5/modeling_qwen3_5.py.  RMSNorm: fp32 statistics,
// x * rsqrt(mean(x^2) + eps) * (1 + w), one rounding to bf16.  Rounding points
// mirror the BF16 torch modules so the pipeline tracks the reference bit for bit
// up to accumulation order.
#include "common.cuh"

namespace kb {
namespace {

// One warp per row of H elements: lane holds H/32 values as H/(32*VEC) chunks
// of VEC consecutive elements (VEC = 8 -> 16-byte accesses; 4 -> 8-byte).
template <int H>
struct RowMap {
  static constexpr int EPL = H / 32;
  static constexpr int VEC = EPL >= 8 ? 8 : EPL;
  static constexpr int CHUNKS = EPL / VEC;
  __device__ static int col(int c, int j) { return c * 32 * VEC + (threadIdx.x & 31) * VEC + j; }
};

template <int H>
__device__ __forceinline__ void load_row(const __nv_bfloat16* p, float (&v)[H / 32]) {
  using M = RowMap<H>;
#pragma unroll
  for (int c = 0; c < M::CHUNKS; ++c) {
    __nv_bfloat162 h[M::VEC / 2];
    if constexpr (M::VEC == 8) {
      *reinterpret_cast<uint4*>(h) = *reinterpret_cast<const uint4*>(p + M::col(c, 0));
    } else {
      *reinterpret_cast<uint2*>(h) = *reinterpret_cast<const uint2*>(p + M::col(c, 0));
    }
#pragma unroll
    for (int j = 0; j < M::VEC / 2; ++j) {
      v[c * M::VEC + 2 * j] = __low2float(h[j]);
      v[c * M::VEC + 2 * j + 1] = __high2float(h[j]);
    }
  }
}

template <int H>
__device__ __forceinline__ void store_row(__nv_bfloat16* p, const float (&v)[H / 32]) {
  using M = RowMap<H>;
#pragma unroll
  for (int c = 0; c < M::CHUNKS; ++c) {
    __nv_bfloat162 h[M::VEC / 2];
#pragma unroll
    for (int j = 0; j < M::VEC / 2; ++j) h[j] = __floats2bfloat162_rn(v[c * M::VEC + 2 * j], v[c * M::VEC + 2 * j + 1]);
    if constexpr (M::VEC == 8) {
      *reinterpret_cast<uint4*>(p + M::col(c, 0)) = *reinterpret_cast<uint4*>(h);
    } else {
      *reinterpret_cast<uint2*>(p + M::col(c, 0)) = *reinterpret_cast<uint2*>(h);
    }
  }
}

template <int H>
__device__ __forceinline__ void rms_row(const float (&x)[H / 32], const float* w, float eps, float (&out)[H / 32]) {
  using M = RowMap<H>;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < H / 32; ++i) ss += x[i] * x[i];
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / float(H) + eps);
#pragma unroll
  for (int c = 0; c < M::CHUNKS; ++c) {
    float wv[M::VEC];
    if constexpr (M::VEC == 8) {  // weights 16-byte aligned (checked by the launcher)
      const float4 w0 = *reinterpret_cast<const float4*>(w + M::col(c, 0));
      const float4 w1 = *reinterpret_cast<const float4*>(w + M::col(c, 4));
      wv[0] = w0.x; wv[1] = w0.y; wv[2] = w0.z; wv[3] = w0.w;
      wv[4] = w1.x; wv[5] = w1.y; wv[6] = w1.z; wv[7] = w1.w;
    } else {
#pragma unroll
      for (int j = 0; j < M::VEC; ++j) wv[j] = w[M::col(c, j)];
    }
#pragma unroll
    for (int j = 0; j < M::VEC; ++j) out[c * M::VEC + j] = (x[c * M::VEC + j] * inv) * (1.0f + wv[j]);
  }
}

template <int H>
__global__ void __launch_bounds__(256) embed_rmsnorm_kernel(const int64_t* ids, int ids_per_row_stride,
                                                            const __nv_bfloat16* table, int64_t vocab,
                                                            const float* w, float eps, __nv_bfloat16* x,
                                                            __nv_bfloat16* normed, int64_t rows) {
  const int64_t r = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  int64_t id = ids[r];
  id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
  float v[H / 32], o[H / 32];
  load_row<H>(table + id * H, v);
  store_row<H>(x + r * H, v);
  rms_row<H>(v, w, eps, o);
  store_row<H>(normed + r * H, o);
}

template <int H>
__global__ void __launch_bounds__(256, H <= 1024 ? 4 : 2) add_rmsnorm_kernel(__nv_bfloat16* x, const __nv_bfloat16* delta,
                                                          int64_t ld_delta, const float* w, float eps,
                                                          __nv_bfloat16* normed, int64_t rows, int64_t row_step,
                                                          int64_t row_offset) {
  // grid-stride over rows: the launcher sizes the grid to the resident CTAs (no partial last wave)
  for (int64_t i = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5); i < rows; i += int64_t(gridDim.x) * 8) {
    const int64_t r = i * row_step + row_offset;  // residual row (normed is written densely at i)
    float v[H / 32], d[H / 32], o[H / 32];
    load_row<H>(x + r * H, v);
    if (delta) {
      load_row<H>(delta + r * ld_delta, d);
#pragma unroll
      for (int j = 0; j < H / 32; ++j) v[j] = bf16r(v[j] + d[j]);
      store_row<H>(x + r * H, v);
    }
    rms_row<H>(v, w, eps, o);
    store_row<H>(normed + i * H, o);
  }
}

// grid (x: 512-column spans, y: rows with stride); each thread two 8-column chunks.
// SiLU through the approximate exp2 / reciprocal units in fp32 pairs.
__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* gu, int64_t ld, int inter,
                                                       __nv_bfloat16* out, int64_t rows) {
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const __nv_bfloat16* g = gu + r * ld;
    const __nv_bfloat16* u = g + inter;
    __nv_bfloat16* o = out + r * int64_t(inter);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = (blockIdx.x * 512 + h * 256 + threadIdx.x) * 8;
      if (c >= inter) continue;
      const uint4 gv = *reinterpret_cast<const uint4*>(g + c);
      const uint4 uv = *reinterpret_cast<const uint4*>(u + c);
      const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gv);
      const uint32_t* uw = reinterpret_cast<const uint32_t*>(&uv);
      uint4 ov;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&ov);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = silu2(bf2f(gw[j]));
        ow[j] = bf2_pack_f2(mul2(bf2f(bf2_pack(a.x, a.y)), bf2f(uw[j])));
      }
      *reinterpret_cast<uint4*>(o + c) = ov;
    }
  }
}

// One warp per (row, head).  D elements per head, EPL = D / 32 per lane (contiguous).
template <int D>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    const __nv_bfloat16* proj, int64_t ld_proj, int Hq, int HK, const float* qw, const float* kw, float eps,
    const __nv_bfloat16* cos_tab, const __nv_bfloat16* sin_tab, int rot, const int64_t* pos_of_row,
    int64_t pos_base, int64_t rows_per_seq, __nv_bfloat16* q_out, int64_t sq_row, int64_t sq_h,
    __nv_bfloat16* k_out, int64_t sk_seq, int64_t sk_pos, int64_t sk_h, __nv_bfloat16* v_out, int64_t sv_seq,
    int64_t sv_pos, int64_t sv_h, int64_t rows) {
  constexpr int EPL = D / 32;
  const int heads = Hq + 2 * HK;
  const int64_t item = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (item >= rows * heads) return;
  const int64_t r = item / heads;
  const int h = int(item % heads);
  const int lane = threadIdx.x & 31;
  // row r = (sequence s, position-in-sequence p); prefill: s = request; decode: s = beam row
  const int64_t s = r / rows_per_seq, p = r % rows_per_seq;
  const int64_t pos = pos_base + (pos_of_row ? pos_of_row[r] : p);
  const __nv_bfloat16* src;
  if (h < Hq) src = proj + r * ld_proj + int64_t(h) * 2 * D;             // q of head h (gate follows it)
  else if (h < Hq + HK) src = proj + r * ld_proj + int64_t(Hq) * 2 * D + int64_t(h - Hq) * D;
  else src = proj + r * ld_proj + int64_t(Hq) * 2 * D + int64_t(HK) * D + int64_t(h - Hq - HK) * D;
  float v[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) v[e] = __bfloat162float(src[lane * EPL + e]);
  if (h >= Hq + HK) {  // value: plain copy into the cache / suffix layout
    const int hk = h - Hq - HK;
    __nv_bfloat16* dst = v_out + s * sv_seq + p * sv_pos + hk * sv_h + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; ++e) dst[e] = __float2bfloat16_rn(v[e]);
    return;
  }
  const float* w = h < Hq ? qw : kw;
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) ss += v[e] * v[e];
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / float(D) + eps);
#pragma unroll
  for (int e = 0; e < EPL; ++e) v[e] = bf16r((v[e] * inv) * (1.0f + w[lane * EPL + e]));
  // partial rotary: dims [0, rot) rotate with the partner half rot/2 away
  const int half = rot / 2;
  const int partner = half / EPL;  // lane distance (half % EPL == 0 checked on the host)
  float pv[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) pv[e] = __shfl_xor_sync(0xffffffffu, v[e], partner);
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const int d = lane * EPL + e;
    if (d < rot) {
      const float c = __bfloat162float(cos_tab[pos * rot + d]);
      const float sn = __bfloat162float(sin_tab[pos * rot + d]);
      const float rh = d < half ? -pv[e] : pv[e];  // rotate_half
      v[e] = bf16r(bf16r(v[e] * c) + bf16r(rh * sn));
    }
  }
  __nv_bfloat16* dst;
  if (h < Hq) dst = q_out + r * sq_row + int64_t(h) * sq_h + lane * EPL;
  else dst = k_out + s * sk_seq + p * sk_pos + int64_t(h - Hq) * sk_h + lane * EPL;
#pragma unroll
  for (int e = 0; e < EPL; ++e) dst[e] = __float2bfloat16_rn(v[e]);
}

// Head dim 256 with 16-byte rows: one warp per (row, head), 8 consecutive
// elements (one 16-byte access) per lane, 32-bit index arithmetic.  Same
// arithmetic and rounding points as qk_norm_rope_kernel.  Eight CTAs per SM (32
// registers): each warp has one row in flight, so the resident warps bound the
// bytes in flight (8 CTAs: 125 us vs 134 us at 5 for the 32 x 1024-row prompt).
// Head dim 256 with 64 rotary dims (the Qwen3.5 attention): lane l holds dims 64 j + 2 l
// and 64 j + 2 l + 1 (j = 0..3), so every lane owns two of the rotary dims (j = 0) and
// their rotate_half partners sit 16 lanes away.  The grid is (head, block of 32 rows):
// each warp takes 4 consecutive rows of one head, so the head's offset, its norm
// weights (1 + w) and the row's sequence / position are set up once and stepped, and
// the next row's loads are in flight while a row is normalised.  Same roundings as
// qk_norm_rope_d256_kernel.
constexpr int kQkRowsPerWarp = 4;
__global__ void __launch_bounds__(256, 5) qk_norm_rope_d256_r64_kernel(
    const __nv_bfloat16* proj, int64_t ld_proj, int Hq, int HK, const float* qw, const float* kw, float eps,
    const __nv_bfloat16* cos_tab, const __nv_bfloat16* sin_tab, const int64_t* pos_of_row, int64_t pos_base,
    int rows_per_seq, __nv_bfloat16* q_out, int64_t sq_row, int64_t sq_h, __nv_bfloat16* k_out, int64_t sk_seq,
    int64_t sk_pos, int64_t sk_h, __nv_bfloat16* v_out, int64_t sv_seq, int64_t sv_pos, int64_t sv_h,
    uint32_t rows) {
  constexpr int D = 256, kRot = 64;
  const int h = int(blockIdx.x);
  const uint32_t r0 = (blockIdx.y * 8u + (threadIdx.x >> 5)) * uint32_t(kQkRowsPerWarp);
  if (r0 >= rows) return;  // whole warps leave together
  const int n = int(min(uint32_t(kQkRowsPerWarp), rows - r0));
  const int lane = threadIdx.x & 31;
  uint32_t s = r0 / uint32_t(rows_per_seq), p = r0 - s * uint32_t(rows_per_seq);  // stepped per row below
  int hoff;  // the head's columns in the projection row
  if (h < Hq) hoff = h * 2 * D;  // q of head h (its gate follows it)
  else if (h < Hq + HK) hoff = Hq * 2 * D + (h - Hq) * D;
  else hoff = Hq * 2 * D + HK * D + (h - Hq - HK) * D;
  const __nv_bfloat16* src = proj + int64_t(r0) * ld_proj + hoff;
  if (h >= Hq + HK) {  // value: plain copy into the cache / suffix layout
    __nv_bfloat16* dst = v_out + (h - Hq - HK) * sv_h + lane * 8;
    for (int i = 0; i < n; ++i) {
      const uint4 raw = *reinterpret_cast<const uint4*>(src + int64_t(i) * ld_proj + lane * 8);
      *reinterpret_cast<uint4*>(dst + s * sv_seq + p * sv_pos) = raw;
      if (++p == uint32_t(rows_per_seq)) {
        p = 0;
        ++s;
      }
    }
    return;
  }
  float w1[8];  // 1 + w of this lane's dims
  {
    const float* w = (h < Hq ? qw : kw) + 2 * lane;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 wj = *reinterpret_cast<const float2*>(w + 64 * j);
      w1[2 * j] = 1.0f + wj.x;
      w1[2 * j + 1] = 1.0f + wj.y;
    }
  }
  auto row_pos = [&](int i, uint32_t pp) -> int64_t {
    return pos_base + (pos_of_row ? pos_of_row[r0 + i] : int64_t(pp));
  };
  uint32_t rw[4], cw, sw;
  {  // row 0's loads
#pragma unroll
    for (int j = 0; j < 4; ++j) rw[j] = *reinterpret_cast<const uint32_t*>(src + 64 * j + 2 * lane);
    const int64_t pos = row_pos(0, p);
    cw = *reinterpret_cast<const uint32_t*>(cos_tab + pos * kRot + 2 * lane);
    sw = *reinterpret_cast<const uint32_t*>(sin_tab + pos * kRot + 2 * lane);
  }
  for (int i = 0; i < n; ++i) {
    const uint32_t ps = s, pp = p;  // this row's sequence / position
    if (++p == uint32_t(rows_per_seq)) {
      p = 0;
      ++s;
    }
    uint32_t nrw[4] = {0u, 0u, 0u, 0u}, ncw = 0u, nsw = 0u;
    if (i + 1 < n) {  // the next row's loads, in flight while this row is computed
      const __nv_bfloat16* nsrc = src + int64_t(i + 1) * ld_proj;
#pragma unroll
      for (int j = 0; j < 4; ++j) nrw[j] = *reinterpret_cast<const uint32_t*>(nsrc + 64 * j + 2 * lane);
      const int64_t npos = row_pos(i + 1, p);
      ncw = *reinterpret_cast<const uint32_t*>(cos_tab + npos * kRot + 2 * lane);
      nsw = *reinterpret_cast<const uint32_t*>(sin_tab + npos * kRot + 2 * lane);
    }
    float v[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = bf2f(rw[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += v[e] * v[e];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / float(D) + eps);
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // bf16 rounding of each pair in one packed conversion
      const float2 nv = bf2f(bf2_pack((v[2 * j] * inv) * w1[2 * j], (v[2 * j + 1] * inv) * w1[2 * j + 1]));
      v[2 * j] = nv.x;
      v[2 * j + 1] = nv.y;
    }
    {  // rotary dims 2 l, 2 l + 1: partner half 32 dims (16 lanes) away
      const float p0 = __shfl_xor_sync(0xffffffffu, v[0], 16), p1 = __shfl_xor_sync(0xffffffffu, v[1], 16);
      const bool lo = lane < 16;
      const float2 c = bf2f(cw), sn = bf2f(sw);
      const float q0 = lo ? -p0 : p0, q1 = lo ? -p1 : p1;          // rotate_half
      const float2 vc = bf2f(bf2_pack(v[0] * c.x, v[1] * c.y));    // bf16(x cos)
      const float2 rs = bf2f(bf2_pack(q0 * sn.x, q1 * sn.y));      // bf16(rotate_half(x) sin)
      const float2 sum = bf2f(bf2_pack(vc.x + rs.x, vc.y + rs.y));
      v[0] = sum.x;
      v[1] = sum.y;
    }
    __nv_bfloat16* dst = h < Hq ? q_out + int64_t(r0 + i) * sq_row + h * sq_h
                                : k_out + ps * sk_seq + pp * sk_pos + (h - Hq) * sk_h;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint32_t*>(dst + 64 * j + 2 * lane) = bf2_pack(v[2 * j], v[2 * j + 1]);
#pragma unroll
    for (int j = 0; j < 4; ++j) rw[j] = nrw[j];
    cw = ncw;
    sw = nsw;
  }
}

__global__ void __launch_bounds__(256, 8) qk_norm_rope_d256_kernel(
    const __nv_bfloat16* proj, int64_t ld_proj, int Hq, int HK, const float* qw, const float* kw, float eps,
    const __nv_bfloat16* cos_tab, const __nv_bfloat16* sin_tab, int rot, const int64_t* pos_of_row,
    int64_t pos_base, int rows_per_seq, __nv_bfloat16* q_out, int64_t sq_row, int64_t sq_h,
    __nv_bfloat16* k_out, int64_t sk_seq, int64_t sk_pos, int64_t sk_h, __nv_bfloat16* v_out, int64_t sv_seq,
    int64_t sv_pos, int64_t sv_h, uint32_t items) {
  constexpr int D = 256;
  const int heads = Hq + 2 * HK;
  const uint32_t item = blockIdx.x * 8u + (threadIdx.x >> 5);
  if (item >= items) return;  // whole warps leave together
  const uint32_t r = item / uint32_t(heads);
  const int h = int(item - r * uint32_t(heads));
  const int lane = threadIdx.x & 31;
  const uint32_t s = r / uint32_t(rows_per_seq), p = r - s * uint32_t(rows_per_seq);
  const int64_t pos = pos_base + (pos_of_row ? pos_of_row[r] : int64_t(p));
  const __nv_bfloat16* src = proj + int64_t(r) * ld_proj;
  if (h < Hq) src += h * 2 * D;  // q of head h (its gate follows it)
  else if (h < Hq + HK) src += Hq * 2 * D + (h - Hq) * D;
  else src += Hq * 2 * D + HK * D + (h - Hq - HK) * D;
  const uint4 raw = *reinterpret_cast<const uint4*>(src + lane * 8);
  if (h >= Hq + HK) {  // value: plain copy into the cache / suffix layout
    *reinterpret_cast<uint4*>(v_out + s * sv_seq + p * sv_pos + (h - Hq - HK) * sv_h + lane * 8) = raw;
    return;
  }
  const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
  float v[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = bf2f(rw[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) ss += v[e] * v[e];
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / float(D) + eps);
  const float* w = (h < Hq ? qw : kw) + lane * 8;
  const float4 w0 = *reinterpret_cast<const float4*>(w), w1 = *reinterpret_cast<const float4*>(w + 4);
  const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {  // bf16 rounding of each pair in one packed conversion
    const float2 n = bf2f(bf2_pack((v[2 * j] * inv) * (1.0f + wv[2 * j]), (v[2 * j + 1] * inv) * (1.0f + wv[2 * j + 1])));
    v[2 * j] = n.x;
    v[2 * j + 1] = n.y;
  }
  // partial rotary: dims [0, rot) rotate with the partner half rot/2 away (rot/2 % 8 == 0)
  const int half = rot / 2;
  float pv[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) pv[e] = __shfl_xor_sync(0xffffffffu, v[e], half / 8);
  if (lane * 8 < rot) {
    const uint4 cr = *reinterpret_cast<const uint4*>(cos_tab + pos * rot + lane * 8);
    const uint4 sr = *reinterpret_cast<const uint4*>(sin_tab + pos * rot + lane * 8);
    const uint32_t cw[4] = {cr.x, cr.y, cr.z, cr.w}, sw[4] = {sr.x, sr.y, sr.z, sr.w};
    const bool lo = lane * 8 < half;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 c = bf2f(cw[j]), sn = bf2f(sw[j]);
      const float r0 = lo ? -pv[2 * j] : pv[2 * j], r1 = lo ? -pv[2 * j + 1] : pv[2 * j + 1];  // rotate_half
      const float2 vc = bf2f(bf2_pack(v[2 * j] * c.x, v[2 * j + 1] * c.y));  // bf16(x cos)
      const float2 rs = bf2f(bf2_pack(r0 * sn.x, r1 * sn.y));                // bf16(rotate_half(x) sin)
      const float2 sum = bf2f(bf2_pack(vc.x + rs.x, vc.y + rs.y));
      v[2 * j] = sum.x;
      v[2 * j + 1] = sum.y;
    }
  }
  __nv_bfloat16* dst = h < Hq ? q_out + int64_t(r) * sq_row + h * sq_h + lane * 8
                              : k_out + s * sk_seq + p * sk_pos + (h - Hq) * sk_h + lane * 8;
  *reinterpret_cast<uint4*>(dst) =
      make_uint4(bf2_pack(v[0], v[1]), bf2_pack(v[2], v[3]), bf2_pack(v[4], v[5]), bf2_pack(v[6], v[7]));
}

}  // namespace
}  // namespace kb

using namespace kb;

// dst row i = src row (i / group) * src_group + index[i] (clamped into the group), 16 bytes a thread.
__global__ void __launch_bounds__(256) gather_rows_kernel(const unsigned char* src, int64_t ld_src,
                                                          const int32_t* index, int group, int src_group,
                                                          int64_t rows, int chunks, unsigned char* dst,
                                                          int64_t ld_dst) {
  const int64_t total = rows * chunks;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i = e / chunks;
    const int c = int(e - i * chunks);
    const int p = min(max(index[i], 0), src_group - 1);
    const int64_t r = (i / group) * src_group + p;
    reinterpret_cast<uint4*>(dst + i * ld_dst)[c] = reinterpret_cast<const uint4*>(src + r * ld_src)[c];
  }
}

extern "C" int kadllm_embed_rmsnorm(const int64_t* ids, const void* table, int64_t vocab, const float* weight,
                                    float eps, void* x, void* normed, int64_t rows, int64_t hidden, void* stream) {
  KB_REQUIRE(rows >= 1 && vocab >= 1, KADLLM_EINVAL, "embed: empty");
  KB_REQUIRE(ids && table && weight && x && normed, KADLLM_EINVAL, "embed: null pointer");
  KB_REQUIRE(((reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(x) |
               reinterpret_cast<uintptr_t>(normed)) & 15) == 0,
             KADLLM_EINVAL, "embed: table, weight and outputs must be 16-byte aligned");
  const unsigned grid = unsigned((rows + 7) / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto T = static_cast<const __nv_bfloat16*>(table);
  auto X = static_cast<__nv_bfloat16*>(x);
  auto N = static_cast<__nv_bfloat16*>(normed);
  if (hidden == 1024) embed_rmsnorm_kernel<1024><<<grid, 256, 0, s>>>(ids, 1, T, vocab, weight, eps, X, N, rows);
  else if (hidden == 2048) embed_rmsnorm_kernel<2048><<<grid, 256, 0, s>>>(ids, 1, T, vocab, weight, eps, X, N, rows);
  else if (hidden == 256) embed_rmsnorm_kernel<256><<<grid, 256, 0, s>>>(ids, 1, T, vocab, weight, eps, X, N, rows);
  else if (hidden == 512) embed_rmsnorm_kernel<512><<<grid, 256, 0, s>>>(ids, 1, T, vocab, weight, eps, X, N, rows);
  else if (hidden == 128) embed_rmsnorm_kernel<128><<<grid, 256, 0, s>>>(ids, 1, T, vocab, weight, eps, X, N, rows);
  else {
    set_error("embed: hidden size %lld not in {128, 256, 512, 1024, 2048}", (long long)hidden);
    return KADLLM_EUNSUPPORTED;
  }
  KB_CHECK_LAUNCH("embed launch");
  return KADLLM_OK;
}

extern "C" int kadllm_add_rmsnorm(void* x, const void* delta, int64_t ld_delta, const float* weight, float eps,
                                  void* normed, int64_t rows, int64_t row_step, int64_t row_offset, int64_t hidden,
                                  void* stream) {
  KB_REQUIRE(x && weight && normed && rows >= 1 && row_step >= 1, KADLLM_EINVAL, "add_rmsnorm: bad arguments");
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  KB_REQUIRE(al16(x) && al16(normed) && al16(weight) && (delta == nullptr || (al16(delta) && ld_delta % 8 == 0)),
             KADLLM_EINVAL, "add_rmsnorm: rows and weights must be 16-byte aligned");
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      sms = 148;
  }
  // resident CTAs of 256 threads: 4 per SM (<= 64 registers) up to hidden 1024, else 2
  const int64_t want = (rows + 7) / 8, resident = int64_t(sms) * (hidden <= 1024 ? 4 : 2);
  const unsigned grid = unsigned(want < resident ? want : resident);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto X = static_cast<__nv_bfloat16*>(x);
  auto Dl = static_cast<const __nv_bfloat16*>(delta);
  auto N = static_cast<__nv_bfloat16*>(normed);
#define KB_NORM_CASE(HH)                                                                                  \
  if (hidden == HH) {                                                                                     \
    add_rmsnorm_kernel<HH><<<grid, 256, 0, s>>>(X, Dl, ld_delta, weight, eps, N, rows, row_step, row_offset); \
    KB_CHECK_LAUNCH("add_rmsnorm launch");                                                                \
    return KADLLM_OK;                                                                                     \
  }
  KB_NORM_CASE(1024)
  KB_NORM_CASE(2048)
  KB_NORM_CASE(256)
  KB_NORM_CASE(512)
  KB_NORM_CASE(128)
#undef KB_NORM_CASE
  set_error("add_rmsnorm: hidden size %lld not in {128, 256, 512, 1024, 2048}", (long long)hidden);
  return KADLLM_EUNSUPPORTED;
}

extern "C" int kadllm_silu_mul(const void* gate_up, int64_t ld, int64_t inter, void* out, int64_t rows,
                               void* stream) {
  KB_REQUIRE(gate_up && out && rows >= 1 && inter % 8 == 0 && ld % 8 == 0, KADLLM_EINVAL,
             "silu_mul: bad arguments (intermediate size and stride must be multiples of 8)");
  KB_REQUIRE(inter < (int64_t(1) << 30) && (reinterpret_cast<uintptr_t>(gate_up) & 15) == 0 &&
                 (reinterpret_cast<uintptr_t>(out) & 15) == 0,
             KADLLM_EINVAL, "silu_mul: pointers must be 16-byte aligned");
  const dim3 grid(unsigned((inter / 8 + 511) / 512), unsigned(rows < 65535 ? rows : 65535));
  silu_mul_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(gate_up), ld, int(inter), static_cast<__nv_bfloat16*>(out), rows);
  KB_CHECK_LAUNCH("silu_mul launch");
  return KADLLM_OK;
}

extern "C" int kadllm_qk_norm_rope(const void* proj, int64_t ld_proj, int64_t q_heads, int64_t kv_heads,
                                   int64_t head_dim, const float* q_weight, const float* k_weight, float eps,
                                   const void* cos_tab, const void* sin_tab, int64_t rotary_dim,
                                   const int64_t* pos_of_row, int64_t pos_base, int64_t rows_per_seq, void* q_out,
                                   int64_t sq_row, int64_t sq_h, void* k_out, int64_t sk_seq, int64_t sk_pos,
                                   int64_t sk_h, void* v_out, int64_t sv_seq, int64_t sv_pos, int64_t sv_h,
                                   int64_t rows, void* stream) {
  KB_REQUIRE(proj && q_weight && k_weight && cos_tab && sin_tab && q_out && k_out && v_out, KADLLM_EINVAL,
             "qk_norm_rope: null pointer");
  KB_REQUIRE(rows >= 1 && rows_per_seq >= 1 && q_heads >= 1 && kv_heads >= 1, KADLLM_EINVAL, "qk_norm_rope: empty");
  const int epl = int(head_dim / 32);
  KB_REQUIRE(rotary_dim % 2 == 0 && rotary_dim <= head_dim && epl >= 1 && (rotary_dim / 2) % epl == 0, KADLLM_EINVAL,
             "qk_norm_rope: rotary_dim/2 must be a multiple of head_dim/32");
  const int64_t items = rows * (q_heads + 2 * kv_heads);
  const unsigned grid = unsigned((items + 7) / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto P = static_cast<const __nv_bfloat16*>(proj);
  auto C = static_cast<const __nv_bfloat16*>(cos_tab);
  auto S = static_cast<const __nv_bfloat16*>(sin_tab);
  auto Q = static_cast<__nv_bfloat16*>(q_out);
  auto K = static_cast<__nv_bfloat16*>(k_out);
  auto Vv = static_cast<__nv_bfloat16*>(v_out);
  const auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  if (head_dim == 256 && rotary_dim == 64 && rows <= 32ll * 65535 && rows_per_seq < (1ll << 31) && al16(proj) &&
      ld_proj % 8 == 0 && al16(q_out) && al16(k_out) && al16(v_out) && al16(q_weight) && al16(k_weight) &&
      al16(cos_tab) && al16(sin_tab) && sq_row % 8 == 0 && sq_h % 8 == 0 && sk_seq % 8 == 0 && sk_pos % 8 == 0 &&
      sk_h % 8 == 0 && sv_seq % 8 == 0 && sv_pos % 8 == 0 && sv_h % 8 == 0) {
    const dim3 g2(unsigned(q_heads + 2 * kv_heads), unsigned((rows + 8 * kQkRowsPerWarp - 1) / (8 * kQkRowsPerWarp)));
    qk_norm_rope_d256_r64_kernel<<<g2, 256, 0, s>>>(P, ld_proj, int(q_heads), int(kv_heads), q_weight, k_weight, eps,
                                                     C, S, pos_of_row, pos_base, int(rows_per_seq), Q, sq_row, sq_h,
                                                     K, sk_seq, sk_pos, sk_h, Vv, sv_seq, sv_pos, sv_h,
                                                     uint32_t(rows));
    KB_CHECK_LAUNCH("qk_norm_rope launch");
    return KADLLM_OK;
  }
  if (head_dim == 256 && items < (1ll << 31) && rows_per_seq < (1ll << 31) && al16(proj) && ld_proj % 8 == 0 &&
      al16(q_out) && al16(k_out) && al16(v_out) && al16(q_weight) && al16(k_weight) && al16(cos_tab) &&
      al16(sin_tab) && sq_row % 8 == 0 && sq_h % 8 == 0 && sk_seq % 8 == 0 && sk_pos % 8 == 0 && sk_h % 8 == 0 &&
      sv_seq % 8 == 0 && sv_pos % 8 == 0 && sv_h % 8 == 0 && (rotary_dim / 2) % 8 == 0 && rotary_dim % 8 == 0) {
    qk_norm_rope_d256_kernel<<<grid, 256, 0, s>>>(P, ld_proj, int(q_heads), int(kv_heads), q_weight, k_weight, eps, C,
                                                  S, int(rotary_dim), pos_of_row, pos_base, int(rows_per_seq), Q,
                                                  sq_row, sq_h, K, sk_seq, sk_pos, sk_h, Vv, sv_seq, sv_pos, sv_h,
                                                  uint32_t(items));
    KB_CHECK_LAUNCH("qk_norm_rope launch");
    return KADLLM_OK;
  }
#define KB_QK_CASE(DD)                                                                                          \
  if (head_dim == DD) {                                                                                         \
    qk_norm_rope_kernel<DD><<<grid, 256, 0, s>>>(P, ld_proj, int(q_heads), int(kv_heads), q_weight, k_weight, eps, \
                                                 C, S, int(rotary_dim), pos_of_row, pos_base, rows_per_seq, Q,      \
                                                 sq_row, sq_h, K, sk_seq, sk_pos, sk_h, Vv, sv_seq, sv_pos, sv_h,   \
                                                 rows);                                                             \
    KB_CHECK_LAUNCH("qk_norm_rope launch");                                                                     \
    return KADLLM_OK;                                                                                           \
  }
  KB_QK_CASE(256)
  KB_QK_CASE(128)
  KB_QK_CASE(64)
  KB_QK_CASE(32)
#undef KB_QK_CASE
  set_error("qk_norm_rope: head_dim %lld not in {32, 64, 128, 256}", (long long)head_dim);
  return KADLLM_EUNSUPPORTED;
}

extern "C" int kadllm_gather_rows(const void* src, int64_t ld_src, const int32_t* index, int64_t group,
                                  int64_t src_group, int64_t rows, int64_t row_bytes, void* dst, int64_t ld_dst,
                                  void* stream) {
  KB_REQUIRE(src && index && dst, KADLLM_EINVAL, "gather rows: null pointer");
  KB_REQUIRE(rows >= 1 && group >= 1 && src_group >= 1 && row_bytes >= 16 && row_bytes % 16 == 0 &&
                 ld_src % 16 == 0 && ld_dst % 16 == 0 && ld_src >= row_bytes && ld_dst >= row_bytes &&
                 group < (int64_t(1) << 30) && src_group < (int64_t(1) << 30) && row_bytes < (int64_t(1) << 30),
             KADLLM_EINVAL, "gather rows: sizes and strides must be positive multiples of 16 bytes");
  KB_REQUIRE(((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0, KADLLM_EINVAL,
             "gather rows: pointers must be 16-byte aligned");
  const int chunks = int(row_bytes / 16);
  const int64_t total = rows * chunks;
  const unsigned blocks = unsigned(total / 256 + 1 < 4096 ? total / 256 + 1 : 4096);
  gather_rows_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const unsigned char*>(src), ld_src, index, int(group), int(src_group), rows, chunks,
      static_cast<unsigned char*>(dst), ld_dst);
  KB_CHECK_LAUNCH("gather rows launch");
  return KADLLM_OK;
}
