// Depthwise causal conv1d replay from a shared prefix (beam decode).
//
// Semantics: src/kadllm/ops.py:166-226 (causal_conv1d) and the Triton kernel
// src/kadllm/kernels/causal_conv1d.py:10-48: each beam row r of request
// r / W convolves the last (width-1) taps of the request's conv state followed
// by its own T suffix columns, then applies SiLU.  fp32 accumulation, one
// rounding to the output dtype.  The state is only read.
//
// HBM-bound; see the tile comment on the kernel for the access pattern.
#include "common.cuh"

namespace kb {
namespace {

constexpr int kMaxWidth = 8;

struct ConvArgs {
  const void* x; int64_t xs0, xs1, xs2;
  const void* state; int64_t ss0, ss1, ss2; int hist;
  const void* weight; const void* bias;
  void* out;
  int dtype, BW, W, C, T, width, silu;
};

// One CTA = (beam row, 32 channels, 64 time steps).  The input window (tile plus
// width-1 steps of history, taken from the request's conv state before t = 0) is
// staged in shared memory with the access order matching x's fastest stride, and
// the [BW, C, T] output is written along time, so both sides are coalesced.
constexpr int kCT = 32, kTT = 64;

__global__ void __launch_bounds__(256) conv_replay_kernel(const ConvArgs a) {
  __shared__ float sx[kCT][kTT + kMaxWidth];
  __shared__ float sy[kCT][kTT + 1];
  const int r = blockIdx.x;
  const int c0 = blockIdx.y * kCT;
  const int t0 = blockIdx.z * kTT;
  const int req = r / a.W;
  const int halo = a.width - 1;
  const int span = kTT + halo;
  const bool chan_fast = a.xs1 == 1;
  for (int i = threadIdx.x; i < kCT * span; i += blockDim.x) {
    const int ci = chan_fast ? i % kCT : i / span;
    const int ti = chan_fast ? i / kCT : i % span;
    const int c = c0 + ci, t = t0 + ti - halo;
    float v = 0.f;
    if (c < a.C && t < a.T) {
      if (t >= 0)
        v = load_as_float(a.x, r * a.xs0 + c * a.xs1 + int64_t(t) * a.xs2, a.dtype);
      else
        v = load_as_float(a.state, req * a.ss0 + c * a.ss1 + int64_t(a.hist + t) * a.ss2, a.dtype);
    }
    sx[ci][ti] = v;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kCT * kTT; i += blockDim.x) {
    const int ci = i / kTT, tt = i % kTT;
    const int c = c0 + ci;
    if (c >= a.C) continue;
    float acc = a.bias ? load_as_float(a.bias, c, a.dtype) : 0.f;
    for (int j = 0; j < a.width; ++j) acc += sx[ci][tt + j] * load_as_float(a.weight, int64_t(c) * a.width + j, a.dtype);
    sy[ci][tt] = a.silu ? silu_f(acc) : acc;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kCT * kTT; i += blockDim.x) {
    const int ci = i / kTT, tt = i % kTT;
    const int c = c0 + ci, t = t0 + tt;
    if (c < a.C && t < a.T) store_from_float(a.out, (int64_t(r) * a.C + c) * a.T + t, a.dtype, sy[ci][tt]);
  }
}

// BF16 with channels contiguous in x (x = proj.transpose(1, 2), the reference's
// layout, xs1 == 1): one CTA = (beam row, 64 channels, 64 steps).  The 64 + 3
// time rows of 128 bytes are staged with 16-byte cp.async copies (the request's
// conv state supplies the rows before t = 0); each thread then runs one channel
// over 16 steps with the 4-tap window in registers and writes its 16 outputs as
// two 16-byte stores along time (the output is [BW, C, T], time contiguous).
constexpr int kFC = 64, kFT = 64, kFRows = kFT + 3, kFPad = kFC + 8;

__global__ void __launch_bounds__(256) conv_bf16_chfast_kernel(const ConvArgs a) {
  __shared__ __align__(16) __nv_bfloat16 sx[kFRows][kFPad];
  const int r = blockIdx.x;
  const int c0 = blockIdx.y * kFC;
  const int t0 = blockIdx.z * kFT;
  const int req = r / a.W;
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(a.x);
  const __nv_bfloat16* st = static_cast<const __nv_bfloat16*>(a.state);
  for (int i = threadIdx.x; i < kFRows * (kFC / 8); i += blockDim.x) {
    const int row = i / (kFC / 8), ch = (i % (kFC / 8)) * 8;
    const int t = t0 - 3 + row, c = c0 + ch;
    __nv_bfloat16* dst = &sx[row][ch];
    if (c >= a.C || t >= a.T) {
      *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
    } else if (t >= 0) {
      cp_async16(dst, x + r * a.xs0 + c + int64_t(t) * a.xs2);
    } else {  // before the suffix: the last taps of the request's conv state (width 4: 3 of them)
#pragma unroll
      for (int e = 0; e < 8; ++e)
        dst[e] = c + e < a.C ? st[req * a.ss0 + (c + e) * a.ss1 + int64_t(a.hist + t) * a.ss2] : __float2bfloat16_rn(0.f);
    }
  }
  cp_async_commit();
  const int ci = threadIdx.x & (kFC - 1), seg = threadIdx.x / kFC;  // channel, 16-step segment
  const int c = c0 + ci;
  float w0 = 0.f, w1 = 0.f, w2 = 0.f, w3 = 0.f, bias = 0.f;
  if (c < a.C) {
    const __nv_bfloat16* wp = static_cast<const __nv_bfloat16*>(a.weight) + int64_t(c) * 4;
    w0 = __bfloat162float(wp[0]); w1 = __bfloat162float(wp[1]);
    w2 = __bfloat162float(wp[2]); w3 = __bfloat162float(wp[3]);
    if (a.bias) bias = __bfloat162float(static_cast<const __nv_bfloat16*>(a.bias)[c]);
  }
  cp_async_wait<0>();
  __syncthreads();
  if (c >= a.C) return;
  const int s0 = seg * 16;  // first output step of this thread (tile-local)
  float xm3 = __bfloat162float(sx[s0][ci]), xm2 = __bfloat162float(sx[s0 + 1][ci]);
  float xm1 = __bfloat162float(sx[s0 + 2][ci]);
  uint32_t packed[8];
#pragma unroll
  for (int k = 0; k < 16; k += 2) {
    const float xa = __bfloat162float(sx[s0 + 3 + k][ci]), xb = __bfloat162float(sx[s0 + 4 + k][ci]);
    float2 y = make_float2(fmaf(w3, xa, fmaf(w2, xm1, fmaf(w1, xm2, fmaf(w0, xm3, bias)))),
                           fmaf(w3, xb, fmaf(w2, xa, fmaf(w1, xm1, fmaf(w0, xm2, bias)))));
    if (a.silu) y = silu2(y);  // exp2 / reciprocal units in pairs, one rounding below
    packed[k / 2] = bf2_pack(y.x, y.y);
    xm3 = xm1; xm2 = xa; xm1 = xb;
  }
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(a.out) + (int64_t(r) * a.C + c) * a.T + t0 + s0;
  const int valid = min(16, a.T - (t0 + s0));
  if (valid == 16 && a.T % 8 == 0) {
    reinterpret_cast<uint4*>(o)[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    reinterpret_cast<uint4*>(o)[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  } else {
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(packed);
    for (int k = 0; k < valid; ++k) o[k] = h[k];
  }
}

}  // namespace
}  // namespace kb

extern "C" int kadllm_causal_conv1d_replay(const void* x, int64_t xs0, int64_t xs1, int64_t xs2,
                                           const void* state, int64_t ss0, int64_t ss1, int64_t ss2,
                                           int64_t hist, const void* weight, const void* bias,
                                           void* out, int dtype, int64_t batch, int64_t beam_width,
                                           int64_t channels, int64_t steps, int64_t width, int silu,
                                           void* stream) {
  using namespace kb;
  KB_REQUIRE(valid_dtype(dtype), KADLLM_EDTYPE, "conv replay: unsupported dtype");
  KB_REQUIRE(batch >= 1 && beam_width >= 1 && channels >= 1 && steps >= 1 && width >= 1, KADLLM_EINVAL,
             "conv replay: empty dimensions");
  KB_REQUIRE(width <= kMaxWidth, KADLLM_EUNSUPPORTED, "conv replay: width %lld > %d", (long long)width, kMaxWidth);
  KB_REQUIRE(hist >= width - 1, KADLLM_EINVAL, "conv replay: state shorter than width-1");
  KB_REQUIRE(batch * beam_width <= 2147483647ll && channels <= 2147483647ll, KADLLM_EINVAL, "conv replay: too large");
  KB_REQUIRE(x && state && weight && out, KADLLM_EINVAL, "conv replay: null pointer");
  ConvArgs a{x, xs0, xs1, xs2, state, ss0, ss1, ss2, int(hist), weight, bias, out, dtype,
             int(batch * beam_width), int(beam_width), int(channels), int(steps), int(width), silu};
  KB_REQUIRE((channels + kCT - 1) / kCT <= 65535 && (steps + kTT - 1) / kTT <= 65535, KADLLM_EINVAL,
             "conv replay: too many channels or steps");
  if (dtype == KADLLM_BF16 && width == 4 && xs1 == 1 && xs2 % 8 == 0 && xs0 % 8 == 0 &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 && steps >= 16) {
    // long suffixes in the reference's channel-contiguous layout: the vectorised sliding window
    dim3 g2(unsigned(batch * beam_width), unsigned((channels + kFC - 1) / kFC), unsigned((steps + kFT - 1) / kFT));
    conv_bf16_chfast_kernel<<<g2, 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
    KB_CHECK_LAUNCH("conv replay launch");
    return KADLLM_OK;
  }
  dim3 grid(unsigned(batch * beam_width), unsigned((channels + kCT - 1) / kCT), unsigned((steps + kTT - 1) / kTT));
  conv_replay_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
  KB_CHECK_LAUNCH("conv replay launch");
  return KADLLM_OK;
}
