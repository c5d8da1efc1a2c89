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
  // First decode step (T = 1): per (beam row, value head) record of the row's delta (fp32)
  // for the next step, or null.  Continuation (T = 2 with proj_prev): the
  // previous step's records (indexed like proj_prev), or null to replay both tokens.
  unsigned char* save;
  const unsigned char* saved;
};

// True when the staged kernel takes this call: D in {64, 128}, T <= 2,
// 16-byte aligned projection rows and output, and a status word.
bool gdn_mixer_staged_ok(const MixerArgs& a);
int gdn_mixer_staged(const MixerArgs& a, cudaStream_t stream);
// Bytes of the first-step records of `rows` beam rows (kadllm_gdn_mixer_record_bytes).
int64_t gdn_mixer_record_bytes(int64_t rows, int64_t v_heads, int64_t dim);

}  // namespace kb
