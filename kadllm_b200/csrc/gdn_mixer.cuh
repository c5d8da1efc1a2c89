// Staged GDN decode mixer (see gdn_mixer.cu): the fast path of
// kadllm_gdn_mixer_replay for head dims 64 / 128 and one or two suffix tokens.
#pragma once
#include "common.cuh"

namespace kb {

struct MixerArgs {
  const __nv_bfloat16* proj;  // [B*W*T, ld_proj] packed projection rows: q | k | v | z | b | a
  int64_t ld_proj;
  const __nv_bfloat16* conv_state;  // [B, conv_dim, conv_hist]
  int64_t conv_hist;
  const __nv_bfloat16* conv_weight;  // [conv_dim, 4]
  const __nv_bfloat16* state;        // [B, HV, D, D] shared recurrent state (K rows, V columns)
  const float* a_log;
  const float* dt_bias;
  const float* norm_weight;
  float norm_eps;
  __nv_bfloat16* out;  // [B*W*T, HV*D]; continuation: [B*W, HV*D] (the new token only)
  int B, W, T, H, HV, D;
  float scale;
  // Continuation (T = 2): token 0 of beam j is the previous step's token of beam parent[b*W + j],
  // whose projection row is proj_prev[b*Wp + parent]; proj holds the new tokens' rows [B*W]
  const __nv_bfloat16* proj_prev;  // [B*Wp, ld_proj] or null
  const int32_t* parent;           // [B*W]
  int Wp;
  uint32_t* status;  // device status word: bit 0 set when a tensor-core wait timed out
};

// True when the staged kernel takes this call: D in {64, 128}, T <= 2,
// 16-byte aligned projection rows and output, and a status word.
bool gdn_mixer_staged_ok(const MixerArgs& a);
int gdn_mixer_staged(const MixerArgs& a, cudaStream_t stream);

}  // namespace kb
