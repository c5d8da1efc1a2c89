// Layout of the beam-selection workspace, shared by the selection kernels
// (beam_select.cu) and the LM-head GEMM that writes its per-chunk statistics
// (gemm_tc.cu).
#pragma once
#include "common.cuh"

namespace kb {
namespace sel {

constexpr int kRowBins = 2048;     // (max - x) in [0, 64) nats, last bin = farther
constexpr int kReqBins = 4096;
constexpr float kBinsPerNat = 32.f;
constexpr int kCap = 16384;        // candidates kept per request
constexpr int kStatThreads = 1024;
constexpr int kStatSlots = 48;     // vectors per thread (V <= 48 * 8 * 1024) for the table
constexpr int kSumMax = kStatSlots * 32;  // 512-byte chunks (256 BF16) per row: chunk c = elements [256 c, 256 c + 256)
constexpr int kChunk = 256;        // elements per chunk

struct Workspace {
  // The flag word sits at offset 0 whatever the widths: the steps of one search
  // (whose previous widths differ) and the status query all find it there.
  // `base` bytes are required; the chunk-maximum summary after them (up to `total`) is optional:
  // without it collect reads whole rows.  `fused` adds the per-chunk sums of exp(x - chunk max)
  // that the LM-head GEMM writes for the fused selection.
  size_t rowstat, rowlen, rowhist, thresh, count, flags, cand, vsum, base, total, tsum, fused;
  Workspace(int64_t B, int64_t Wp) {
    auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
    const int64_t rows = B * Wp;
    flags = 0;
    rowstat = al(flags + sizeof(uint32_t));
    rowlen = al(rowstat + rows * sizeof(float2));
    rowhist = al(rowlen + rows * sizeof(uint32_t));
    thresh = al(rowhist + rows * kRowBins * sizeof(uint32_t));
    count = al(thresh + B * sizeof(float));
    cand = al(count + B * sizeof(uint32_t));
    vsum = base = al(cand + B * kCap * sizeof(unsigned long long));
    total = al(vsum + rows * kSumMax * sizeof(uint16_t));
    tsum = total;
    fused = al(tsum + rows * kSumMax * sizeof(float));
  }
};

}  // namespace sel
}  // namespace kb
