// Depthwise causal conv1d replay from a shared prefix (beam decode).
//
// Semantics: src/kadllm/ops.py:166-226 (causal_conv1d) and the Triton kernel
// src/kadllm/kernels/causal_conv1d.py:10-48: each beam row r of request
// r / W convolves the last (width-1) taps of the request's conv state followed
// by its own T suffix columns, then applies SiLU.  fp32 accumulation, one
// rounding to the output dtype.  The state is only read.
//
// HBM-bound: one thread per (beam row, channel) walks the T columns keeping
// the sliding window in registers; channels are the fastest-varying index so
// reads of the (typically channel-contiguous) projection are coalesced.
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

__global__ void __launch_bounds__(256) conv_replay_kernel(const ConvArgs a) {
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  const int r = blockIdx.x;
  if (c >= a.C) return;
  const int req = r / a.W;
  float w[kMaxWidth], win[kMaxWidth];
  for (int j = 0; j < a.width; ++j) w[j] = load_as_float(a.weight, int64_t(c) * a.width + j, a.dtype);
  // window[0 .. width-2] = last width-1 prefix taps
  for (int j = 0; j < a.width - 1; ++j)
    win[j] = load_as_float(a.state, req * a.ss0 + c * a.ss1 + int64_t(a.hist - (a.width - 1) + j) * a.ss2, a.dtype);
  const float bias = a.bias ? load_as_float(a.bias, c, a.dtype) : 0.f;
  for (int t = 0; t < a.T; ++t) {
    const float xt = load_as_float(a.x, r * a.xs0 + c * a.xs1 + int64_t(t) * a.xs2, a.dtype);
    win[a.width - 1] = xt;
    float acc = bias;
    for (int j = 0; j < a.width; ++j) acc += win[j] * w[j];
    const float o = a.silu ? silu_f(acc) : acc;
    store_from_float(a.out, (int64_t(r) * a.C + c) * a.T + t, a.dtype, o);
    for (int j = 0; j + 1 < a.width; ++j) win[j] = win[j + 1];
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
  const int threads = 256;
  KB_REQUIRE((channels + threads - 1) / threads <= 65535, KADLLM_EINVAL, "conv replay: too many channels");
  dim3 grid(unsigned(batch * beam_width), unsigned((channels + threads - 1) / threads));
  conv_replay_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  KB_CHECK_LAUNCH("conv replay launch");
  return KADLLM_OK;
}
