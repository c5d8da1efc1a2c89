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
  dim3 grid(unsigned(batch * beam_width), unsigned((channels + kCT - 1) / kCT), unsigned((steps + kTT - 1) / kTT));
  conv_replay_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
  KB_CHECK_LAUNCH("conv replay launch");
  return KADLLM_OK;
}
