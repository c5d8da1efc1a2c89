// Per-request beam selection over the full vocabulary (one GRBeam step).
//
// Semantics: src/kadllm/grbeam.py:75-104.  For request b with Wp parent beams
// and vocabulary V:  logp = log_softmax(float(logits[b, w, :]))  (over the full,
// unmasked row), masked entries -> -inf (no renormalisation), score = logp +
// parent_score[b, w]; keep the top `width` of the Wp*V candidates, sorted by
// score; parent = idx // V, token = idx % V; the new history is the parent's
// history followed by the token.  Each score is evaluated in the reference's
// fp32 order ((x - max) - log(sum)) + parent.  Ties are broken by the lower flat
// index (torch.topk leaves their order unspecified).
//
// The reference loops over requests on the host (32 launches of a 254 MB
// temporary each).  Here the whole batch is four launches and no temporary of
// logits size:
//   1. rowstats   per row: max and sum-exp, and a 2048-bin histogram of
//                 (max - x) in 1/32-nat bins (BF16 without a mask: of the
//                 16-byte vectors' maxima, lower bounds of the element counts);
//   2. threshold  per request: shifts every row histogram by the row's score
//                 offset into a request histogram and picks the highest score
//                 threshold that provably keeps >= width candidates above it;
//   3. collect    per row that can reach the threshold: appends candidates >=
//                 threshold (score, flat index) to a per-request buffer, reading
//                 only the 512-byte chunks whose maximum (a summary rowstats
//                 writes when the workspace has room for it) reaches it;
//   4. finalize   per request: bitonic sort of the buffer (score desc, index
//                 asc), writes scores and the gathered history.
// Buffers live in a caller-provided workspace (kadllm_beam_select_workspace).
#include <mutex>
#include <type_traits>

#include "beam_select.cuh"

namespace kb {
namespace {

using namespace sel;
constexpr int kRowThreads = 512;
constexpr float kLog2e = 1.4426950408889634f;

struct SelArgs {
  const void* logits; int dtype; int64_t ld;
  const float* parent;         // [B*Wp] or null (zeros)
  const uint8_t* mask;         // [B*Wp, V] or null
  const int64_t* old_hist;     // [B*Wp, depth] or null
  float* out_scores;           // [B*W]
  int64_t* out_hist;           // [B*W, depth+1]
  int32_t* out_parent;         // [B*W] previous-beam index of each selected beam, or null
  float2* rowstat;             // [rows] (max, log-sum-exp offset)
  uint32_t* rowhist;           // [rows, kRowBins]
  uint32_t* rowlen;            // [rows] leading bins of rowhist that can be non-zero
  float* thresh;               // [B]
  uint32_t* count;             // [B]
  uint32_t* flags;             // [1] bit 0: candidate overflow
  unsigned long long* cand;    // [B, kCap]
  uint16_t* vsum;              // [rows, kSumMax] bf16 maximum of each 32-vector chunk, or null
  const float* tsum;           // [rows, kSumMax] sum of exp(x - chunk max) per chunk (fused selection), or null
  int B, Wp, W, depth;
  int64_t V;
};

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// Visit every element of a row: f(index, value).  Uses 16-byte loads when the
// row is 16-byte aligned and V is a multiple of the vector width.
template <typename T, typename F>
__device__ __forceinline__ void for_row(const T* row, int64_t V, bool vec, F&& f) {
  constexpr int N = 16 / sizeof(T);
  if (vec) {
    for (int64_t i = int64_t(threadIdx.x) * N; i < V; i += int64_t(blockDim.x) * N) {
      const uint4 u = *reinterpret_cast<const uint4*>(row + i);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < N; ++j) f(i + j, to_f<T>(e[j]));
    }
  } else {
    for (int64_t i = threadIdx.x; i < V; i += blockDim.x) f(i, to_f<T>(row[i]));
  }
}

__device__ float block_reduce(float v, bool is_max, float* red) {
  v = is_max ? warp_max(v) : warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float x = lane < nw ? red[lane] : (is_max ? -INFINITY : 0.f);
    x = is_max ? warp_max(x) : warp_sum(x);
    if (lane == 0) red[32] = x;
  }
  __syncthreads();
  return red[32];
}

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float order_inv(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

template <typename T>
__global__ void __launch_bounds__(kRowThreads) rowstats_kernel(const SelArgs a, bool vec) {
  __shared__ uint32_t hist[kRowBins];
  __shared__ float red[33];
  const int64_t r = blockIdx.x;
  const T* row = reinterpret_cast<const T*>(a.logits) + r * a.ld;
  float m = -INFINITY;
  for_row<T>(row, a.V, vec, [&](int64_t, float x) { m = fmaxf(m, x); });
  m = block_reduce(m, true, red);
  for (int i = threadIdx.x; i < kRowBins; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const float ml = m * kLog2e;
  const uint8_t* mrow = a.mask ? a.mask + r * a.V : nullptr;
  float s = 0.f;
  for_row<T>(row, a.V, vec, [&](int64_t i, float x) {
    s += exp2f(x * kLog2e - ml);
    if (mrow == nullptr || mrow[i]) {
      const float d = (m - x) * kBinsPerNat;
      const int bin = d < float(kRowBins - 1) ? int(d) : kRowBins - 1;
      atomicAdd(&hist[bin], 1u);
    }
  });
  s = block_reduce(s, false, red);
  if (threadIdx.x == 0) a.rowstat[r] = make_float2(m, logf(s));
  __syncthreads();
  for (int i = threadIdx.x; i < kRowBins; i += blockDim.x) a.rowhist[r * kRowBins + i] = hist[i];
  if (threadIdx.x == 0) a.rowlen[r] = kRowBins - 1;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// BF16 logits without a mask (the decode hot path).  Persistent: one
// 1024-thread CTA per SM loops over rows and reads each row from HBM once.
//   pass 1 (HBM): per-thread running max and sum of exp, packed bf16x2 max per
//     16-byte vector.  The sum is kept relative to a reference value that moves
//     only when a vector's maximum exceeds it by more than kRefSlack nats (the
//     first vector, in practice), so the stream has no divergent rescale;
//   tau: a lower bound on the row's W-th largest value.  Each warp sorts its 32
//     per-thread maxima; the minimum over the n warps of the ceil(W/n)-th
//     largest leaves >= W elements of the row at or above tau.  Only those can
//     be among the request's top W (a row shares parent score and normaliser),
//     so binning only them leaves the threshold bin unchanged, and bins past
//     tau's stay empty (rowlen);
//   pass 2: each thread's 16-byte vector maxima of the row are kept in shared
//     memory (bf16, [slot][thread]) and the maxima at or above tau are binned:
//     d = 32 (max - vmax), one FFMA (bit-identical to (max - vmax) * 32).  A
//     vector whose maximum reaches a score holds at least one candidate at or
//     above it, so these counts are lower bounds of the element counts: the
//     threshold they give still provably keeps >= width candidates (tau bounds
//     >= W thread maxima, each in its own vector), and collect then gathers the
//     elements exactly.  With room in the workspace the same pass records, per
//     warp and slot, the maximum of the warp's 32 vectors (one contiguous
//     512-byte chunk), so collect reads only the chunks that can hold
//     candidates.  Pass 2 of row r runs inside pass 1 of the CTA's next
//     row (two tables and two histograms, alternating), so the logits are read
//     from HBM exactly once.
constexpr float kRefSlack = 64.f;
__host__ __device__ constexpr size_t stat_smem(int slots) { return size_t(2) * slots * kStatThreads * 2; }

// maximum of the 8 bf16 values (NaN ignored, like fmaxf)
__device__ __forceinline__ __nv_bfloat16 vec_max_bf(const uint4& u) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  const __nv_bfloat162 t = __hmax2(__hmax2(h[0], h[1]), __hmax2(h[2], h[3]));
  return __hmax(__low2bfloat16(t), __high2bfloat16(t));
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&x)[8]) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    x[2 * j] = __uint_as_float(w[j] << 16);
    x[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
  }
}

// Per-thread running max and sum of exp2(x log2e - ref log2e), the sum kept as a
// pair (even / odd elements) in packed fp32x2 arithmetic.  ref <= m and
// (m - ref) <= kRefSlack, so no term exceeds 2^93.
struct OnlineSum {
  float m = -INFINITY, ref = -INFINITY, rl = 0.f;
  float2 s = make_float2(0.f, 0.f);
  // accumulate one 16-byte vector; returns its maximum
  __device__ __forceinline__ __nv_bfloat16 add(const uint4& u) {
    const __nv_bfloat16 hb = vec_max_bf(u);
    const float hi = __bfloat162float(hb);
    m = fmaxf(m, hi);
    if (hi > ref + kRefSlack) {  // the first finite vector, or a jump of more than kRefSlack nats
      const float c = ex2_approx((ref - hi) * kLog2e);
      s = mul2(s, make_float2(c, c));
      ref = hi;
      rl = hi * kLog2e;
    }
    const float2 l2e = make_float2(kLog2e, kLog2e), nrl = make_float2(-rl, -rl);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 t = fma2(bf2f(w[j]), l2e, nrl);
      s = add2(s, make_float2(ex2_approx(t.x), ex2_approx(t.y)));
    }
    return hb;
  }
  // the sum relative to `to` (>= ref)
  __device__ __forceinline__ float sum_at(float to) const {
    return ref == -INFINITY ? 0.f : (s.x + s.y) * ex2_approx((ref - to) * kLog2e);
  }
};

__global__ void __launch_bounds__(kStatThreads, 1) rowstats_bf16_kernel(const SelArgs a) {
  __shared__ uint32_t hists[2][kRowBins];  // alternating rows: binned during the next row, exported after it
  __shared__ float red[2 * 96];
  extern __shared__ __align__(16) unsigned char dsm[];
  __nv_bfloat16* vmax = reinterpret_cast<__nv_bfloat16*>(dsm);  // [2][slots][nt] vector maxima
  constexpr int nt = kStatThreads, nwarps = kStatThreads / 32;
  const int rows = a.B * a.Wp;  // < 2^31 (checked by the host)
  const int nvec = int(a.V / 8);
  const int slots = (nvec + nt - 1) / nt;
  const int tid = threadIdx.x, lane = tid & 31;
  for (int j = tid; j < 2 * kRowBins; j += nt) hists[j / kRowBins][j % kRowBins] = 0;
  for (int j = tid; j < 2 * slots * nt / 8; j += nt)  // table entries past the row's vectors stay -inf
    reinterpret_cast<uint4*>(vmax)[j] = make_uint4(0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u);
  __syncthreads();  // before any thread writes its own entries
  // the CTA's previous row, binned while the current one streams in
  int pr = -1;
  float ptau = 0.f, pm32 = 0.f;
  int pbin = 0;
  bool pact = false;
  int par = 0;  // table and histogram of the current row
  const __nv_bfloat16* base = reinterpret_cast<const __nv_bfloat16*>(a.logits);
  // the first four vectors of the CTA's next row, loaded before the current row's
  // reductions so HBM keeps streaming through them
  uint4 f0, f1, f2, f3;
  const bool full4 = tid + 3 * nt < nvec;
  if (full4 && int(blockIdx.x) < rows) {
    const uint4* r0 = reinterpret_cast<const uint4*>(base + int64_t(blockIdx.x) * a.ld);
    f0 = r0[tid]; f1 = r0[tid + nt]; f2 = r0[tid + 2 * nt]; f3 = r0[tid + 3 * nt];
  }
  for (int r = blockIdx.x;; r += gridDim.x, par ^= 1) {
    const bool cur = r < rows;
    const uint4* row = reinterpret_cast<const uint4*>(base + int64_t(cur ? r : 0) * a.ld);
    __nv_bfloat16* tcur = vmax + size_t(par) * slots * nt + tid;
    const __nv_bfloat16* tprev = vmax + size_t(par ^ 1) * slots * nt + tid;
    uint32_t* phist = hists[par ^ 1];  // the previous row's bins
    uint16_t* psum = a.vsum && pr >= 0 ? a.vsum + int64_t(pr) * kSumMax : nullptr;
    // previous row's vector at slot k (present: inside the row): bin its maximum if it reaches tau
    auto bin_prev = [&](int k, bool present) {
      if (present && pact) {
        const float v = __bfloat162float(tprev[k * nt]);
        if (v >= ptau) atomicAdd(&phist[int(fminf(fmaf(v, -kBinsPerNat, pm32), float(kRowBins - 1)))], 1u);
      }
    };
    OnlineSum acc;
    const int wfirst = tid - lane;  // the warp's first thread: loops below are warp-uniform
    if (cur) {
      int k = 0;
      for (; wfirst + (k + 3) * nt + 31 < nvec; k += 4) {  // four 16-byte HBM loads in flight
        const int i = tid + k * nt;
        uint4 u0 = f0, u1 = f1, u2 = f2, u3 = f3;  // first batch: prefetched
        if (k) {
          u0 = row[i]; u1 = row[i + nt]; u2 = row[i + 2 * nt]; u3 = row[i + 3 * nt];
        }
        if (pr >= 0) {
          bin_prev(k, true);
          bin_prev(k + 1, true);
          bin_prev(k + 2, true);
          bin_prev(k + 3, true);
        }
        tcur[k * nt] = acc.add(u0);
        tcur[(k + 1) * nt] = acc.add(u1);
        tcur[(k + 2) * nt] = acc.add(u2);
        tcur[(k + 3) * nt] = acc.add(u3);
      }
      for (; wfirst + k * nt < nvec; ++k) {
        const int i = tid + k * nt;
        const bool has = i < nvec;
        if (has) tcur[k * nt] = acc.add(row[i]);
        if (pr >= 0) bin_prev(k, has);
      }
    } else if (pr >= 0) {
      for (int k = 0; wfirst + k * nt < nvec; ++k) bin_prev(k, tid + k * nt < nvec);
    }
    if (psum) {  // the previous row's chunk maxima, from its table (intact until the barrier below):
      // chunk (slot k, warp w) = table entries [k][32 w, 32 w + 32), one chunk per thread, the
      // four 16-byte reads rotated so that a warp's reads spread over all banks
      const __nv_bfloat16* tb = vmax + size_t(par ^ 1) * slots * nt;
      for (int c = tid; c < slots * 32; c += nt) {
        const uint4* src = reinterpret_cast<const uint4*>(tb + (c >> 5) * nt + (c & 31) * 32);
        __nv_bfloat162 m2 = __bfloat162bfloat162(__ushort_as_bfloat16(0xff80u));
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const uint4 u = src[(jj + (c >> 1)) & 3];
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
          m2 = __hmax2(m2, __hmax2(__hmax2(h[0], h[1]), __hmax2(h[2], h[3])));
        }
        psum[c] = __bfloat16_as_ushort(__hmax(__low2bfloat16(m2), __high2bfloat16(m2)));  // NaN ignored
      }
    }
    // one exchange per row: each warp publishes its maximum, its sum rescaled to that
    // maximum and its ceil(W/n)-th largest thread maximum; every thread combines the 32
    float m = -INFINITY, sum = 0.f, tau = -INFINITY, mt = -INFINITY;
    if (cur) {
      if (full4 && r + int(gridDim.x) < rows) {  // next row's first batch, in flight during the reductions
        const uint4* rn = reinterpret_cast<const uint4*>(base + int64_t(r + gridDim.x) * a.ld);
        f0 = rn[tid]; f1 = rn[tid + nt]; f2 = rn[tid + 2 * nt]; f3 = rn[tid + 3 * nt];
      }
      mt = acc.m;
      const float wm = warp_max(mt);
      const float ws = warp_sum(acc.sum_at(wm));
      float wk = -INFINITY;
      if (a.W <= 32 * nwarps) {
        const int kth = (a.W + nwarps - 1) / nwarps - 1;
        float v = mt;
#pragma unroll
        for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
          for (int j = k >> 1; j > 0; j >>= 1) {
            const float o = __shfl_xor_sync(0xffffffffu, v, j);
            v = (((lane & j) == 0) == ((lane & k) == 0)) ? fmaxf(v, o) : fminf(v, o);
          }
        }
        wk = __shfl_sync(0xffffffffu, v, kth);
      }
      float* xr = red + (par ? 96 : 0);  // alternate rows: readers of one row never meet writers of the next
      if (lane == 0) {
        xr[tid >> 5] = wm;
        xr[32 + (tid >> 5)] = ws;
        xr[64 + (tid >> 5)] = wk;
      }
    }
    // every thread has streamed this row and binned the previous one
    __syncthreads();
    if (pr >= 0) {  // export the previous row's bins and clear them (binned into again two rows on)
      const int len = min(pbin + 1, kRowBins - 1);
      if (tid == 0) a.rowlen[pr] = uint32_t(len);
      for (int j = tid; j <= pbin; j += nt) {
        if (j < len) a.rowhist[int64_t(pr) * kRowBins + j] = phist[j];
        phist[j] = 0;
      }
    }
    if (!cur) break;
    {  // every warp combines the 32 entries in parallel, lane w taking warp w's (nwarps == 32)
      static_assert(nwarps == 32, "one entry per lane");
      const float* xr = red + (par ? 96 : 0);
      const float mw = xr[lane];
      m = warp_max(mw);
      sum = warp_sum(mw == -INFINITY ? 0.f : xr[32 + lane] * ex2_approx((mw - m) * kLog2e));
      if (a.W <= 32 * nwarps) {
        float k = xr[64 + lane];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) k = fminf(k, __shfl_xor_sync(0xffffffffu, k, o));
        tau = k;
      }
    }
    if (tid == 0) a.rowstat[r] = make_float2(m, logf(sum));
    pr = r;
    ptau = tau;
    pm32 = m * kBinsPerNat;
    // tau's bin bounds every binned element's; -inf, NaN (all -inf row) -> last bin
    pbin = int(fminf(fmaf(tau, -kBinsPerNat, pm32), float(kRowBins - 1)));
    pact = mt >= tau;
  }
}

// Row statistics from the per-chunk statistics the LM-head GEMM wrote (fused selection):
// one warp per row combines the chunk maxima (vsum) and sums (tsum) into the row's
// max and log-sum-exp, and bins the chunk maxima -- each one an element of its chunk,
// so the counts are lower bounds of the element counts, as with the 16-byte
// vectors' maxima of rowstats_bf16_kernel -- into the row histogram, skipping the
// chunks below a bound on the row's W-th largest chunk maximum (32 lanes x the
// ceil(W/32)-th largest of each lane's maxima).
constexpr int kTileStatWarps = 8;
constexpr int kTopPerLane = 8;

__global__ void __launch_bounds__(kTileStatWarps * 32) tile_rowstats_kernel(const SelArgs a, int nchunk) {
  extern __shared__ uint32_t hsm[];  // [kTileStatWarps][kRowBins]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows = int64_t(a.B) * a.Wp;
  const int64_t r = int64_t(blockIdx.x) * kTileStatWarps + warp;
  if (r >= rows) return;  // whole warp; no block-wide barrier below
  uint32_t* hist = hsm + warp * kRowBins;
  const uint16_t* vs = a.vsum + r * kSumMax;
  const float* ts = a.tsum + r * kSumMax;
  float m = -INFINITY;
  for (int c = lane; c < nchunk; c += 32) m = fmaxf(m, __uint_as_float(uint32_t(vs[c]) << 16));
  m = warp_max(m);
  const int K = (a.W + 31) / 32;  // chunk maxima per lane that 32 lanes need to hold >= W of them
  float top[kTopPerLane];
#pragma unroll
  for (int i = 0; i < kTopPerLane; ++i) top[i] = -INFINITY;
  float sum = 0.f;
  for (int c = lane; c < nchunk; c += 32) {
    const float x = __uint_as_float(uint32_t(vs[c]) << 16);
    if (x > -INFINITY) sum = fmaf(ts[c], ex2_approx((x - m) * kLog2e), sum);
    float v = x;  // insert into the lane's descending top list
#pragma unroll
    for (int i = 0; i < kTopPerLane; ++i) {
      const float hi = fmaxf(top[i], v);
      v = fminf(top[i], v);
      top[i] = hi;
    }
  }
  sum = warp_sum(sum);
  float tau = -INFINITY;
  if (K <= kTopPerLane) {
    float k = top[0];
#pragma unroll
    for (int i = 1; i < kTopPerLane; ++i)
      if (i == K - 1) k = top[i];
    for (int o = 16; o > 0; o >>= 1) k = fminf(k, __shfl_xor_sync(0xffffffffu, k, o));
    tau = k;
  }
  if (lane == 0) a.rowstat[r] = make_float2(m, logf(sum));
  const float m32 = m * kBinsPerNat;
  // tau's bin bounds every binned maximum's; -inf, NaN (an all -inf row) -> the last bin
  const int pbin = int(fminf(fmaf(tau, -kBinsPerNat, m32), float(kRowBins - 1)));
  const int len = min(pbin + 1, kRowBins - 1);
  for (int j = lane; j <= pbin; j += 32) hist[j] = 0;
  __syncwarp();
  for (int c = lane; c < nchunk; c += 32) {
    const float x = __uint_as_float(uint32_t(vs[c]) << 16);
    if (x >= tau) atomicAdd(&hist[int(fminf(fmaf(x, -kBinsPerNat, m32), float(kRowBins - 1)))], 1u);
  }
  __syncwarp();
  if (lane == 0) a.rowlen[r] = uint32_t(len);
  for (int j = lane; j < len; j += 32) a.rowhist[r * kRowBins + j] = hist[j];
}

__global__ void __launch_bounds__(1024) threshold_kernel(const SelArgs a) {
  __shared__ uint32_t rh[kReqBins];
  __shared__ float red[33];
  __shared__ uint32_t scan[1024];
  const int b = blockIdx.x;
  // S_ref: best candidate score of the request (score of each row's max element)
  float sref = -INFINITY;
  for (int w = threadIdx.x; w < a.Wp; w += blockDim.x) {
    const float p = a.parent ? a.parent[int64_t(b) * a.Wp + w] : 0.f;
    const float2 st = a.rowstat[int64_t(b) * a.Wp + w];
    sref = fmaxf(sref, p - st.y);
  }
  sref = block_reduce(sref, true, red);
  for (int i = threadIdx.x; i < kReqBins; i += blockDim.x) rh[i] = 0;
  __syncthreads();
  if (sref > -INFINITY) {  // one warp per row: rows are independent, bins few
    const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int w = threadIdx.x >> 5; w < a.Wp; w += nw) {
      const int64_t r = int64_t(b) * a.Wp + w;
      const float p = a.parent ? a.parent[r] : 0.f;
      const float off = p - a.rowstat[r].y;
      if (!(off > -INFINITY)) continue;
      const float e = (sref - off) * kBinsPerNat;
      if (e >= float(kReqBins)) continue;
      const int base = int(e) + 1;
      const int len = min(int(a.rowlen[r]), kReqBins - base);
      for (int j = lane; j < len; j += 32) {
        const uint32_t c = a.rowhist[r * kRowBins + j];
        if (c) atomicAdd(&rh[base + j], c);
      }
    }
  }
  __syncthreads();
  // smallest K with cumulative count >= W: each thread owns 4 consecutive bins
  constexpr int per = kReqBins / 1024;
  uint32_t local = 0;
  for (int j = 0; j < per; ++j) local += rh[threadIdx.x * per + j];
  scan[threadIdx.x] = local;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const uint32_t v = threadIdx.x >= off ? scan[threadIdx.x - off] : 0;
    __syncthreads();
    scan[threadIdx.x] += v;
    __syncthreads();
  }
  __shared__ int found;
  if (threadIdx.x == 0) found = kReqBins;
  __syncthreads();
  uint32_t run = scan[threadIdx.x] - local;
  for (int j = 0; j < per; ++j) {
    run += rh[threadIdx.x * per + j];
    if (run >= uint32_t(a.W)) {
      atomicMin(&found, threadIdx.x * per + j);
      break;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // half a bin of slack absorbs fp32 rounding of the evaluated scores
    a.thresh[b] = (found < kReqBins && sref > -INFINITY)
                      ? sref - (float(found) + 1.5f) / kBinsPerNat
                      : -INFINITY;
    a.count[b] = 0;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) collect_kernel(const SelArgs a, bool vec) {
  const int64_t r = blockIdx.x;
  const int b = int(r / a.Wp), w = int(r % a.Wp);
  const float p = a.parent ? a.parent[r] : 0.f;
  const float2 st = a.rowstat[r];
  const float tau = a.thresh[b];
  if (!(p > -INFINITY) || (p - st.y) < tau) return;  // no candidate of this row reaches tau
  const T* row = reinterpret_cast<const T*>(a.logits) + r * a.ld;
  const uint8_t* mrow = a.mask ? a.mask + r * a.V : nullptr;
  const uint32_t base_idx = uint32_t(int64_t(w) * a.V);
  unsigned long long* out = a.cand + int64_t(b) * kCap;
  if (std::is_same<T, __nv_bfloat16>::value && a.vsum) {
    // only the 512-byte chunks whose maximum reaches tau (the score is monotonic in x)
    const int nvec = int(a.V / 8), nchunk = (nvec + 1023) / 1024 * 32;
    const uint16_t* vs = a.vsum + r * kSumMax;
    const uint4* row4 = reinterpret_cast<const uint4*>(row);
    const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int c0 = (threadIdx.x >> 5) * 32; c0 < nchunk; c0 += nw * 32) {
      bool hit = false;
      const int c = c0 + lane;
      if (c < nchunk && (c >> 5) * 1024 + (c & 31) * 32 < nvec) {  // a chunk holding vectors of the row
        const float x = __uint_as_float(uint32_t(vs[c]) << 16);
        hit = ((x - st.x) - st.y) + p >= tau;
      }
      uint32_t bal = __ballot_sync(0xffffffffu, hit);
      while (bal) {
        const int cc = c0 + __ffs(bal) - 1;
        bal &= bal - 1;
        const int vi = (cc >> 5) * 1024 + (cc & 31) * 32 + lane;
        if (vi < nvec) {
          const uint4 u = row4[vi];
          const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float x = __bfloat162float(e[j]);
            const float score = ((x - st.x) - st.y) + p;
            if (score >= tau && score > -INFINITY) {
              const uint32_t pos = atomicAdd(&a.count[b], 1u);
              if (pos < kCap) {
                const uint32_t idx = base_idx + uint32_t(vi * 8 + j);
                out[pos] = (static_cast<unsigned long long>(order_key(score)) << 32) | (0xffffffffu - idx);
              }
            }
          }
        }
      }
    }
    return;
  }
  for_row<T>(row, a.V, vec, [&](int64_t i, float x) {
    const float score = ((x - st.x) - st.y) + p;
    if (score >= tau && score > -INFINITY && (mrow == nullptr || mrow[i])) {
      const uint32_t pos = atomicAdd(&a.count[b], 1u);
      if (pos < kCap) {
        const uint32_t idx = base_idx + uint32_t(i);
        out[pos] = (static_cast<unsigned long long>(order_key(score)) << 32) | (0xffffffffu - idx);
      }
    }
  });
}

__global__ void __launch_bounds__(1024) finalize_kernel(const SelArgs a) {
  extern __shared__ unsigned long long keys[];
  const int b = blockIdx.x;
  const uint32_t total = a.count[b];
  const int n = int(min(total, uint32_t(kCap)));
  if (total > uint32_t(kCap) && threadIdx.x == 0) atomicOr(a.flags, 1u);
  int N = 1;
  while (N < max(n, a.W)) N <<= 1;
  for (int i = threadIdx.x; i < N; i += blockDim.x) keys[i] = i < n ? a.cand[int64_t(b) * kCap + i] : 0ull;
  __syncthreads();
  // bitonic sort, descending
  for (int k = 2; k <= N; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < N; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long x = keys[i], y = keys[ixj];
          const bool desc = (i & k) == 0;
          if (desc ? (x < y) : (x > y)) {
            keys[i] = y;
            keys[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int w = threadIdx.x; w < a.W; w += blockDim.x) {
    float score = -INFINITY;
    uint32_t idx = 0;
    if (w < n) {
      const unsigned long long k = keys[w];
      score = order_inv(uint32_t(k >> 32));
      idx = 0xffffffffu - uint32_t(k & 0xffffffffull);
    }
    const int64_t parent = int64_t(idx) / a.V, token = int64_t(idx) % a.V;
    const int64_t o = int64_t(b) * a.W + w;
    a.out_scores[o] = score;
    if (a.out_parent) a.out_parent[o] = int32_t(parent);
    int64_t* h = a.out_hist + o * (a.depth + 1);
    const int64_t* src = a.old_hist ? a.old_hist + (int64_t(b) * a.Wp + parent) * a.depth : nullptr;
    for (int d = 0; d < a.depth; ++d) h[d] = src[d];
    h[a.depth] = token;
  }
}

template <typename T>
int launch_select(SelArgs& a, bool vec, cudaStream_t s) {
  const int64_t rows = int64_t(a.B) * a.Wp;
  static int num_sms = 0;
  if (num_sms == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      num_sms = 148;
  }
  const int slots = int((a.V / 8 + kStatThreads - 1) / kStatThreads);
  if (std::is_same<T, __nv_bfloat16>::value && vec && a.mask == nullptr && slots <= kStatSlots && rows < (int64_t(1) << 30)) {
    const size_t smem = stat_smem(slots);
    if (cudaFuncSetAttribute(rowstats_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) !=
        cudaSuccess) {
      set_error("beam select: cannot reserve %zu bytes of shared memory", smem);
      return KADLLM_ECUDA;
    }
    rowstats_bf16_kernel<<<unsigned(rows < num_sms ? rows : num_sms), kStatThreads, smem, s>>>(a);
  } else {
    a.vsum = nullptr;  // only the BF16 kernel writes the chunk summary
    rowstats_kernel<T><<<unsigned(rows), kRowThreads, 0, s>>>(a, vec);
  }
  threshold_kernel<<<a.B, 1024, 0, s>>>(a);
  collect_kernel<T><<<unsigned(rows), 256, 0, s>>>(a, vec);
  int N = 1;
  while (N < max(kCap, a.W)) N <<= 1;
  const size_t smem = size_t(N) * sizeof(unsigned long long);
  if (cudaFuncSetAttribute(finalize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
    set_error("beam select: cannot reserve %zu bytes of shared memory", smem);
    return KADLLM_ECUDA;
  }
  finalize_kernel<<<a.B, 1024, smem, s>>>(a);
  KB_CHECK_LAUNCH("beam select launch");
  return KADLLM_OK;
}

// The fused selection: the LM-head GEMM (kadllm_gemm_logits) already wrote every
// row's chunk maxima and sums into the workspace; no pass over the logits.
int launch_select_fused(SelArgs& a, cudaStream_t s) {
  const int64_t rows = int64_t(a.B) * a.Wp;
  const int nchunk = int((a.V + kChunk - 1) / kChunk);
  const size_t hsmem = size_t(kTileStatWarps) * kRowBins * sizeof(uint32_t);
  if (cudaFuncSetAttribute(tile_rowstats_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(hsmem)) !=
      cudaSuccess) {
    set_error("beam select: cannot reserve %zu bytes of shared memory", hsmem);
    return KADLLM_ECUDA;
  }
  tile_rowstats_kernel<<<unsigned((rows + kTileStatWarps - 1) / kTileStatWarps), kTileStatWarps * 32, hsmem, s>>>(
      a, nchunk);
  threshold_kernel<<<a.B, 1024, 0, s>>>(a);
  collect_kernel<__nv_bfloat16><<<unsigned(rows), 256, 0, s>>>(a, true);
  int N = 1;
  while (N < max(kCap, a.W)) N <<= 1;
  const size_t smem = size_t(N) * sizeof(unsigned long long);
  if (cudaFuncSetAttribute(finalize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess) {
    set_error("beam select: cannot reserve %zu bytes of shared memory", smem);
    return KADLLM_ECUDA;
  }
  finalize_kernel<<<a.B, 1024, smem, s>>>(a);
  KB_CHECK_LAUNCH("beam select launch");
  return KADLLM_OK;
}

}  // namespace
}  // namespace kb

extern "C" int64_t kadllm_beam_select_workspace_fused(int64_t batch, int64_t prev_width) {
  return int64_t(kb::sel::Workspace(batch, prev_width).fused);
}

extern "C" int64_t kadllm_beam_select_workspace(int64_t batch, int64_t prev_width) {
  return int64_t(kb::sel::Workspace(batch, prev_width).total);
}

namespace kb {
namespace {
// Shared body of the selection entry points.  `flags` overrides the workspace's
// flag word when non-null.
int select_with_workspace(const void* logits, int logits_dtype, int64_t ld_row, const float* parent_scores,
                          const void* mask, const int64_t* old_history, float* out_scores, int64_t* out_history,
                          int32_t* out_parent, void* workspace, int64_t workspace_bytes, uint32_t* flags, int64_t batch,
                          int64_t prev_width, int64_t vocab, int64_t width, int64_t depth, void* stream,
                          bool fused = false) {
  KB_REQUIRE(valid_dtype(logits_dtype), KADLLM_EDTYPE, "beam select: unsupported logits dtype");
  KB_REQUIRE(batch >= 1 && prev_width >= 1 && vocab >= 1 && width >= 1 && depth >= 0, KADLLM_EINVAL,
             "beam select: empty dimensions");
  KB_REQUIRE(width <= prev_width * vocab, KADLLM_EINVAL, "beam width exceeds the number of candidate slots");
  KB_REQUIRE(width <= kCap, KADLLM_EUNSUPPORTED, "beam select: width %lld above %d", (long long)width, kCap);
  KB_REQUIRE(prev_width * vocab < 0xffffffffll, KADLLM_EUNSUPPORTED, "beam select: more than 2^32 candidates");
  KB_REQUIRE(batch <= 65535 && batch * prev_width <= 2147483647ll, KADLLM_EINVAL, "beam select: too many rows");
  KB_REQUIRE(ld_row >= vocab, KADLLM_EINVAL, "beam select: row stride shorter than the vocabulary");
  KB_REQUIRE(logits && out_scores && out_history && workspace && (depth == 0 || old_history), KADLLM_EINVAL,
             "beam select: null pointer");
  const Workspace ws(batch, prev_width);
  KB_REQUIRE(workspace_bytes >= int64_t(ws.base), KADLLM_EINVAL, "beam select: workspace too small");
  KB_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, KADLLM_EINVAL,
             "beam select: workspace must be 256-byte aligned");
  char* w = static_cast<char*>(workspace);
  SelArgs a{};
  a.logits = logits; a.dtype = logits_dtype; a.ld = ld_row;
  a.parent = parent_scores; a.mask = static_cast<const uint8_t*>(mask); a.old_hist = old_history;
  a.out_scores = out_scores; a.out_hist = out_history; a.out_parent = out_parent;
  a.rowstat = reinterpret_cast<float2*>(w + ws.rowstat);
  a.rowhist = reinterpret_cast<uint32_t*>(w + ws.rowhist);
  a.rowlen = reinterpret_cast<uint32_t*>(w + ws.rowlen);
  a.thresh = reinterpret_cast<float*>(w + ws.thresh);
  a.count = reinterpret_cast<uint32_t*>(w + ws.count);
  a.flags = flags ? flags : reinterpret_cast<uint32_t*>(w + ws.flags);
  a.cand = reinterpret_cast<unsigned long long*>(w + ws.cand);
  a.vsum = workspace_bytes >= int64_t(ws.total) ? reinterpret_cast<uint16_t*>(w + ws.vsum) : nullptr;
  if (fused) {
    KB_REQUIRE(logits_dtype == KADLLM_BF16 && mask == nullptr && workspace_bytes >= int64_t(ws.fused) &&
                   vocab <= int64_t(kSumMax) * kChunk,
               KADLLM_EINVAL, "fused beam select: BF16 logits without a mask, a fused workspace, V <= %d",
               kSumMax * kChunk);
    a.tsum = reinterpret_cast<const float*>(w + ws.tsum);
  }
  a.B = int(batch); a.Wp = int(prev_width); a.W = int(width); a.depth = int(depth); a.V = vocab;
  const int esz = dtype_size(logits_dtype);
  const int vw = 16 / esz;
  const bool vec = (reinterpret_cast<uintptr_t>(logits) & 15) == 0 && vocab % vw == 0 && ld_row % vw == 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (flags == nullptr && depth == 0) {
    // the first step of a search (no history yet) starts the workspace's flag word afresh
    cudaError_t e = cudaMemsetAsync(a.flags, 0, sizeof(uint32_t), s);
    KB_REQUIRE(e == cudaSuccess, KADLLM_ECUDA, "beam select: %s", cudaGetErrorString(e));
  }
  if (fused) {
    KB_REQUIRE(vec, KADLLM_EINVAL, "fused beam select: logits rows must be 16-byte aligned, V a multiple of 8");
    return launch_select_fused(a, s);
  }
  if (logits_dtype == KADLLM_BF16) return launch_select<__nv_bfloat16>(a, vec, s);
  if (logits_dtype == KADLLM_F16) return launch_select<__half>(a, vec, s);
  return launch_select<float>(a, vec, s);
}
}  // namespace
}  // namespace kb

extern "C" int kadllm_beam_select(const void* logits, int logits_dtype, int64_t ld_row, const float* parent_scores,
                                  const void* mask, const int64_t* old_history, float* out_scores,
                                  int64_t* out_history, int32_t* out_parent, void* workspace,
                                  int64_t workspace_bytes, int64_t batch, int64_t prev_width, int64_t vocab,
                                  int64_t width, int64_t depth, void* stream) {
  return kb::select_with_workspace(logits, logits_dtype, ld_row, parent_scores, mask, old_history, out_scores,
                                   out_history, out_parent, workspace, workspace_bytes, nullptr, batch, prev_width,
                                   vocab, width, depth, stream);
}

extern "C" int kadllm_beam_select_fused(const void* logits, int64_t ld_row, const float* parent_scores,
                                        const int64_t* old_history, float* out_scores, int64_t* out_history,
                                        int32_t* out_parent, void* workspace, int64_t workspace_bytes, int64_t batch,
                                        int64_t prev_width, int64_t vocab, int64_t width, int64_t depth,
                                        void* stream) {
  return kb::select_with_workspace(logits, KADLLM_BF16, ld_row, parent_scores, nullptr, old_history, out_scores,
                                   out_history, out_parent, workspace, workspace_bytes, nullptr, batch, prev_width,
                                   vocab, width, depth, stream, true);
}

extern "C" int kadllm_beam_select_status(const void* workspace, int64_t batch, int64_t prev_width,
                                         uint32_t* flags_out, void* stream) {
  using namespace kb;
  KB_REQUIRE(workspace && flags_out, KADLLM_EINVAL, "beam select status: null pointer");
  const sel::Workspace ws(batch, prev_width);
  cudaError_t e = cudaMemcpyAsync(flags_out, static_cast<const char*>(workspace) + ws.flags, sizeof(uint32_t),
                                  cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  KB_REQUIRE(e == cudaSuccess, KADLLM_ECUDA, "beam select status: %s", cudaGetErrorString(e));
  return KADLLM_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant.  Some callers cannot allocate device memory at the
// point where they select beams: embedded / plugin hosts that hand the library
// only the tensors they own, serving runtimes whose memory budget is fixed
// when the model loads, and allocators that forbid growth on the decode path.
// For them the selection keeps its scratch in one fixed array that lives in
// this library's device image.
//
// kNoAllocScratchBytes (9 MiB) is reserved on every GPU that loads the library,
// until the process exits.  It covers batch * prev_width <= 512 rows and
// batch <= 32 requests (per-row histograms 4 MiB, candidate buffers 4 MiB).
// Every call shares the array and it keeps the previous call's contents: the
// kernels rewrite everything they read except the per-request counters, which
// the threshold kernel clears, so no clearing is needed here -- but two calls
// whose work overlaps on the GPU (for instance on two streams) race on the
// array and must be serialised by the caller.
// ---------------------------------------------------------------------------
namespace kb {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(9) << 20;
static __device__ __align__(256) unsigned char g_select_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mutex;

// The host-side symbol is only a stand-in for the array: its device address is
// resolved once per device, with that device current.
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  KB_REQUIRE(e == cudaSuccess, KADLLM_ECUDA, "beam select (no-alloc): cudaGetDevice: %s", cudaGetErrorString(e));
  KB_REQUIRE(dev >= 0 && dev < kMaxDevices, KADLLM_EUNSUPPORTED, "beam select (no-alloc): device %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_select_scratch);
    KB_REQUIRE(e == cudaSuccess && p != nullptr, KADLLM_ECUDA,
               "beam select (no-alloc): cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return KADLLM_OK;
}

}  // namespace
}  // namespace kb

extern "C" int kadllm_beam_select_noalloc(const void* logits, int logits_dtype, int64_t ld_row,
                                          const float* parent_scores, const void* mask,
                                          const int64_t* old_history, float* out_scores,
                                          int64_t* out_history, uint32_t* out_flags, int64_t batch,
                                          int64_t prev_width, int64_t vocab, int64_t width, int64_t depth,
                                          void* stream) {
  using namespace kb;
  KB_REQUIRE(out_flags, KADLLM_EINVAL, "beam select (no-alloc): null flags pointer");
  KB_REQUIRE(batch >= 1 && prev_width >= 1, KADLLM_EINVAL, "beam select (no-alloc): empty dimensions");
  const sel::Workspace ws(batch, prev_width);
  KB_REQUIRE(ws.base <= kNoAllocScratchBytes && batch <= 32 && batch * prev_width <= 512, KADLLM_EINVAL,
             "beam select (no-alloc): batch %lld x prev_width %lld needs %zu bytes of scratch; the static "
             "maximum is %zu bytes (batch <= 32, batch * prev_width <= 512)",
             (long long)batch, (long long)prev_width, ws.base, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (int rc = scratch_for_current_device(&scratch)) return rc;
  // the caller's flag word replaces the scratch flag word: clear it, the kernels OR into it
  cudaError_t e = cudaMemsetAsync(out_flags, 0, sizeof(uint32_t), static_cast<cudaStream_t>(stream));
  KB_REQUIRE(e == cudaSuccess, KADLLM_ECUDA, "beam select (no-alloc): %s", cudaGetErrorString(e));
  return select_with_workspace(logits, logits_dtype, ld_row, parent_scores, mask, old_history, out_scores,
                               out_history, nullptr, scratch, int64_t(kNoAllocScratchBytes), out_flags, batch,
                               prev_width, vocab, width, depth, stream);
}
