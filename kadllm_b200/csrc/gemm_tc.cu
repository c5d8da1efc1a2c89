// Persistent BF16 GEMM on the 5th-generation tensor cores with the epilogues the
// GRBeam pipeline fuses into its projections:
//
//   C[M, N] = A[M, K] . B[N, K]^T      (torch.nn.functional.linear(A, B); both
//                                       operands K-major, FP32 accumulation; the
//                                       tensor maps fill zeros past M, N and K)
//
// It replaces every plain projection of the Qwen3.5 decoder as the reference
// runs it through Transformers' nn.Linear (src/kadllm/adapters/qwen3_5.py:144-202,
// 226-235: in_proj_*, q/k/v_proj, o_proj, out_proj, the MLP's gate / up / down
// projections and the LM head).
//
// Design (B200, sm_100a):
//  * CTA pairs (2-CTA clusters, tcgen05 cta_group::2): a pair computes a 256 x 256
//    output tile; each CTA stages its 128 rows of A and 128 rows of B per K step
//    (64 BF16 = one 128-byte swizzle row) with tensor-map copies, so every byte of a
//    tile crosses L2 -> SM once per pair.
//  * One CTA per SM (192 threads): warp 0 issues the copies, warp 1 of rank 0 issues
//    the MMAs (M = 256, N = 256, K = 16) and commits each stage back to both CTAs'
//    "empty" barriers, warps 2-5 drain the accumulator.  Six 32 KB stages.  The
//    residual update runs 320 threads: warps 2-9 drain, two per TMEM lane quadrant,
//    with five stages in the shared memory left.
//  * The accumulator is double-buffered in tensor memory (2 x 256 columns), so the
//    epilogue of tile i overlaps the main loop of tile i + 1.  Tiles are spread over
//    the pairs round-robin, grouped 8 M-tiles at a time for L2 reuse of B.
//  * Epilogues: TMEM -> registers -> a 32 x 64 swizzled shared-memory box per warp
//    (two per warp, alternating) -> one tensor-map store per box (coalesced, clipped
//    at the edges); the residual box is fetched by a tensor-map copy into the same box:
//      kStore    C = bf16(acc)
//      kSiluMul  B's rows interleaved in 128-row blocks [gate block j | up block j];
//                C[:, 128 j + i] = bf16(bf16(silu(bf16(gate))) * bf16(up)), the
//                rounding of act_fn(gate_proj(x)) * up_proj(x) in BF16
//      kAddResid C = bf16(resid + bf16(acc)) (the residual update x = x + f(x); C may
//                alias resid)
//  * Every mbarrier wait is bounded; a wait that gives up sets bit 0 of the caller's
//    status word, the kernel drains what it started and frees its tensor memory.
#include <cudaTypedefs.h>

#include <mutex>

#include "beam_select.cuh"
#include "common.cuh"
#include "tcgen05_pair.cuh"

namespace kb {
namespace {

constexpr int kBM = 128;                                // rows of A per CTA (256 per pair)
constexpr int kBN = 256;                                // columns of the pair's tile
constexpr int kBK = 64;                                 // one 128-byte swizzle row of BF16
constexpr uint32_t kABytes = kBM * kBK * 2;             // 16 KB
constexpr uint32_t kBBytes = (kBN / 2) * kBK * 2;       // 16 KB (this CTA's half of B)
constexpr uint32_t kStageBytes = kABytes + kBBytes;     // 32 KB
constexpr int kGroupM = 8;
constexpr long long kWait = 1ll << 31;
constexpr uint32_t kBoxBytes = 32 * 128;                // epilogue staging box: 32 rows x 64 BF16

enum Epilogue { kStore = 0, kSiluMul = 1, kAddResid = 2, kLogits = 3 };

// Per epilogue: drain warps (the residual update: two per TMEM lane quadrant, each
// taking half of the tile's columns, so that the last tile's drain, with its residual
// copies, overlaps nothing for half as long), operand stages in the shared memory
// they leave, threads per CTA.
template <int EPI>
struct Cfg {
  static constexpr int kEpiWarps = EPI == kAddResid ? 8 : 4;
  static constexpr int kStages = EPI == kAddResid ? 5 : 6;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr size_t kSmemBytes =
      1024 + size_t(kStages) * kStageBytes + size_t(kEpiWarps) * 2 * kBoxBytes + 32 * 8 + 128;
};

struct GemmArgs {
  __nv_bfloat16* c;
  int64_t ldc;
  const __nv_bfloat16* resid;
  int64_t ld_resid;
  int M, N, K, n_out;  // N: rows of B (columns of the product); n_out: columns of C
  int tiles_m, tiles_n;
  uint32_t* status;
  uint16_t* vsum;  // kLogits: per (row, 256-column chunk) the BF16 maximum ...
  float* tsum;     // ... and the sum of exp(x - that maximum), rows kSumMax apart
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& tm, int& tn) {
  const int span = kGroupM * tiles_n;
  const int first = (t / span) * kGroupM;
  const int gm = min(kGroupM, tiles_m - first);
  const int r = t % span;
  tm = first + r % gm;
  tn = r / gm;
}

__device__ __forceinline__ void spin_cycles(long long n) {
  const long long t0 = clock64();
  while (clock64() - t0 < n) {
  }
}

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Cfg<EPI>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const __grid_constant__ CUtensorMap map_c, const __grid_constant__ CUtensorMap map_r,
                   const GemmArgs g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kStages = Cfg<EPI>::kStages, kEpiWarps = Cfg<EPI>::kEpiWarps;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(kStages) * kStageBytes + kEpiWarps * 2 * kBoxBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;   // [2] accumulator ready (both CTAs)
  uint64_t* tempty = tfull + 2;        // [2] accumulator drained (rank 0's: 8 warps arrive)
  uint64_t* drain = tempty + 2;        // error path: the MMA issuer's last commit
  uint64_t* rbars = drain + 1;         // [kEpiWarps] epilogue warps' residual-box copies
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbars + kEpiWarps);

  const uint32_t rank = tc2::cta_rank();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = int(tc2::cluster_id()), npairs = int(tc2::num_clusters());
  const int total = g.tiles_m * g.tiles_n;
  const int kblocks = (g.K + kBK - 1) / kBK;  // a partial last block reads zeros past K

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(full + s, 1);
      tc::mbar_init(empty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(tfull + a, 1);
      tc::mbar_init(tempty + a, 2 * kEpiWarps);
    }
    tc::mbar_init(drain, 1);
    for (int w = 0; w < kEpiWarps; ++w) tc::mbar_init(rbars + w, 1);
    tc2::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tc2::prefetch_map(&map_a);
    tc2::prefetch_map(&map_b);
    tc2::prefetch_map(&map_c);
  }
  if (warp == 1) tc2::tmem_alloc(tmem_slot, 512);
  tc::fence_before();
  tc2::cluster_sync();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;

  bool ok = true;
  if (warp == 0) {
    if (lane == 0) {  // copies: this CTA's 128 rows of A and of B per stage
      int s = 0;
      uint32_t ph = 0;
      for (int t = pair; t < total && ok; t += npairs) {
        int tm, tn;
        tile_coords(t, g.tiles_m, g.tiles_n, tm, tn);
        const int arow = tm * 256 + int(rank) * kBM, brow = tn * kBN + int(rank) * (kBN / 2);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!tc::mbar_wait(empty + s, ph ^ 1u, kWait)) {
            ok = false;
            break;
          }
          // rank 0's full barrier counts both CTAs' bytes
          if (rank == 0) tc::mbar_expect_tx(full + s, 2 * kStageBytes);
          const uint32_t bar = tc2::peer_addr(smem_u32(full + s), 0);
          uint8_t* st = smem + size_t(s) * kStageBytes;
          tc2::tma_load_2d(st, &map_a, kb * kBK, arow, bar);
          tc2::tma_load_2d(st + kABytes, &map_b, kb * kBK, brow, bar);
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (ok) {
        // every stage's last release (the issuer's commit, possibly still in flight) arrives
        // before this CTA may exit
        for (int i = 0; i < kStages && ok; ++i) {
          ok = tc::mbar_wait(empty + s, ph ^ 1u, kWait);
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
      } else {
        spin_cycles(1 << 20);  // copies already issued land before the CTA may exit
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {  // the pair's MMA issuer
      const uint32_t idesc = tc::idesc_bf16(256, kBN, 0, 0);
      int s = 0, acc = 0;
      uint32_t ph = 0, acc_ph = 0;
      bool issued = false;
      for (int t = pair; t < total && ok; t += npairs) {
        if (!tc::mbar_wait(tempty + acc, acc_ph ^ 1u, kWait)) {
          ok = false;
          break;
        }
        tc::fence_after();
        const uint32_t d = tmem + uint32_t(acc * kBN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!tc::mbar_wait(full + s, ph, kWait)) {
            ok = false;
            break;
          }
          tc::fence_after();
          const uint32_t a_addr = smem_u32(smem + size_t(s) * kStageBytes);
          const uint64_t ad = tc2::desc_sw128(a_addr), bd = tc2::desc_sw128(a_addr + kABytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)  // +32 bytes per K = 16 slice (+2 in the descriptor's 16-byte units)
            tc2::mma(d, ad + uint64_t(2 * k), bd + uint64_t(2 * k), idesc, kb > 0 || k > 0);
          issued = true;
          tc2::commit(smem_u32(empty + s));                      // this CTA's stage is free
          tc2::commit(tc2::peer_addr(smem_u32(empty + s), 1));   // and the peer's
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        tc2::commit(smem_u32(tfull + acc));
        tc2::commit(tc2::peer_addr(smem_u32(tfull + acc), 1));
        if (++acc == 2) {
          acc = 0;
          acc_ph ^= 1u;
        }
      }
      if (!ok && issued) {  // let the MMAs already issued finish before the memory is released
        tc2::commit(smem_u32(drain));
        tc::mbar_wait(drain, 0, kWait);
      }
    }
  } else {  // warps 2..: epilogue; warp w reads TMEM lanes 32 (w % 4) .. + 31
    const int q = warp & 3, part = (warp - 2) / 4;
    // two 32-row x 64-column staging boxes per warp (128-byte swizzle: chunk j of row r at
    // r * 128 + ((j ^ (r % 8)) * 16)), written from registers and stored by the tensor map
    uint8_t* stage = smem + size_t(kStages) * kStageBytes + size_t(warp - 2) * 2 * kBoxBytes;
    uint64_t* rbar = rbars + (warp - 2);
    constexpr int kOutCols = EPI == kSiluMul ? kBN / 2 : kBN;  // output columns per tile
    constexpr int kPartCols = kOutCols / (kEpiWarps / 4);      // this warp's share of them
    int acc = 0, nbuf = 0;
    uint32_t acc_ph = 0, rph = 0;
    constexpr float kLog2e = 1.4426950408889634f;
    for (int t = pair; t < total && ok; t += npairs) {
      int tm, tn;
      tile_coords(t, g.tiles_m, g.tiles_n, tm, tn);
      if (!tc::mbar_wait(tfull + acc, acc_ph, kWait)) {
        ok = false;
        break;
      }
      tc::fence_after();
      const int row0 = tm * 256 + int(rank) * kBM + q * 32;
      const uint32_t tbase = tc::taddr(tmem, q * 32, acc * kBN);
      float lm = -INFINITY, ls = 0.f;  // kLogits: this row's running chunk maximum and sum
#pragma unroll 1
      for (int c = part * kPartCols; c < (part + 1) * kPartCols && ok; c += 64) {
        const int col = tn * kOutCols + c;
        if (row0 >= g.M || col >= g.n_out) continue;  // warp-uniform: nothing of this box is stored
        uint8_t* buf = stage + (nbuf & 1) * kBoxBytes;
        if (lane == 0) tc2::bulk_wait_read<1>();  // the store issued from this box two boxes ago has read it
        __syncwarp();
        if (EPI == kAddResid && lane == 0) {
          tc::mbar_expect_tx(rbar, kBoxBytes);
          tc2::tma_load_2d_cta(buf, &map_r, col, row0, rbar);
        }
        uint32_t w[32];
        if (EPI == kSiluMul) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t gr[32], ur[32];
            tc::ld32(tbase + uint32_t(c + 32 * h), gr);
            tc::ld32(tbase + uint32_t(kBN / 2 + c + 32 * h), ur);
            tc::wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float2 gate = bf2f(bf2_pack(__uint_as_float(gr[2 * j]), __uint_as_float(gr[2 * j + 1])));
              const float2 up = bf2f(bf2_pack(__uint_as_float(ur[2 * j]), __uint_as_float(ur[2 * j + 1])));
              const float2 a = silu2(gate);
              w[16 * h + j] = bf2_pack_f2(mul2(bf2f(bf2_pack(a.x, a.y)), up));
            }
          }
        } else {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t r[32];
            tc::ld32(tbase + uint32_t(c + 32 * h), r);
            tc::wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j)
              w[16 * h + j] = bf2_pack(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
          }
        }
        if (EPI == kLogits) {  // the BF16-rounded logits of this box into the row's chunk statistics
          const bool full = col + 64 <= g.n_out;
          float bm = -INFINITY;
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            const float2 f = bf2f(w[k]);
            const float x0 = (full || col + 2 * k < g.n_out) ? f.x : -INFINITY;
            const float x1 = (full || col + 2 * k + 1 < g.n_out) ? f.y : -INFINITY;
            bm = fmaxf(bm, fmaxf(x0, x1));
          }
          if (bm > lm) {
            ls = lm == -INFINITY ? 0.f : ls * fast_ex2((lm - bm) * kLog2e);
            lm = bm;
          }
          if (lm > -INFINITY) {
            const float nl = -lm * kLog2e;
            float2 acc2 = make_float2(0.f, 0.f);
#pragma unroll
            for (int k = 0; k < 32; ++k) {
              const float2 f = bf2f(w[k]);
              const float x0 = (full || col + 2 * k < g.n_out) ? f.x : -INFINITY;
              const float x1 = (full || col + 2 * k + 1 < g.n_out) ? f.y : -INFINITY;
              acc2.x += fast_ex2(fmaf(x0, kLog2e, nl));
              acc2.y += fast_ex2(fmaf(x1, kLog2e, nl));
            }
            ls += acc2.x + acc2.y;
          }
        }
        const uint32_t row_addr = smem_u32(buf) + uint32_t(lane) * 128u;
        if (EPI == kAddResid) {
          if (!tc::mbar_wait(rbar, rph, kWait)) ok = false;
          rph ^= 1u;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 x;
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];\n"
                         : "=r"(x.x), "=r"(x.y), "=r"(x.z), "=r"(x.w)
                         : "r"(row_addr + (uint32_t(j ^ (lane & 7)) << 4)));
            w[4 * j] = bf2_pack_f2(add2(bf2f(x.x), bf2f(w[4 * j])));
            w[4 * j + 1] = bf2_pack_f2(add2(bf2f(x.y), bf2f(w[4 * j + 1])));
            w[4 * j + 2] = bf2_pack_f2(add2(bf2f(x.z), bf2f(w[4 * j + 2])));
            w[4 * j + 3] = bf2_pack_f2(add2(bf2f(x.w), bf2f(w[4 * j + 3])));
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(row_addr + (uint32_t(j ^ (lane & 7)) << 4)),
                       "r"(w[4 * j]), "r"(w[4 * j + 1]), "r"(w[4 * j + 2]), "r"(w[4 * j + 3])
                       : "memory");
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tc2::tma_store_2d(&map_c, col, row0, buf);
          tc2::bulk_commit();
        }
        ++nbuf;
      }
      if (EPI == kLogits && row0 + lane < g.M && tn * kBN < g.n_out) {
        const int64_t o = int64_t(row0 + lane) * sel::kSumMax + tn;
        g.vsum[o] = uint16_t(__float_as_uint(lm) >> 16);  // a BF16 value (or -inf): exact
        g.tsum[o] = ls;
      }
      tc::fence_before();
      __syncwarp();
      if (lane == 0) tc2::arrive_cluster(tc2::peer_addr(smem_u32(tempty + acc), 0));
      if (++acc == 2) {
        acc = 0;
        acc_ph ^= 1u;
      }
    }
    if (lane == 0) tc2::bulk_wait_all();  // the stores have read (and written) everything before exit
    __syncwarp();
  }
  if (!ok) atomicOr(g.status, 1u);  // a bounded wait gave up
  __syncwarp();
  tc::fence_before();
  tc2::cluster_sync();
  if (warp == 1) {
    tc::fence_after();
    tc2::tmem_free(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// Host side: tensor maps through the driver entry point (no link against libcuda).
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// rows x cols BF16 matrix, row stride ld elements; boxes of 64 columns x box_rows rows.
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  const cuuint32_t box[2] = {uint32_t(kBK), uint32_t(box_rows)};
  const cuuint32_t elem[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int EPI>
int launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& mr,
           const GemmArgs& g, cudaStream_t s) {
  static int max_pairs[64] = {};
  int dev = 0;
  KB_REQUIRE(cudaGetDevice(&dev) == cudaSuccess && dev < 64, KADLLM_ECUDA, "gemm: no current device");
  if (max_pairs[dev] == 0) {
    KB_REQUIRE(cudaFuncSetAttribute(gemm_tc_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(Cfg<EPI>::kSmemBytes)) == cudaSuccess,
               KADLLM_ECUDA, "gemm: cannot reserve %zu bytes of shared memory", Cfg<EPI>::kSmemBytes);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(Cfg<EPI>::kThreads);
    cfg.dynamicSmemBytes = Cfg<EPI>::kSmemBytes;
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, gemm_tc_kernel<EPI>, &cfg) != cudaSuccess || clusters < 1) {
      cudaGetLastError();
      int sms = 148;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      clusters = sms / 2;
    }
    max_pairs[dev] = clusters;
  }
  const int total = g.tiles_m * g.tiles_n;
  const int pairs = total < max_pairs[dev] ? total : max_pairs[dev];
  gemm_tc_kernel<EPI><<<dim3(2 * pairs), dim3(Cfg<EPI>::kThreads), Cfg<EPI>::kSmemBytes, s>>>(ma, mb, mc, mr, g);
  KB_CHECK_LAUNCH("gemm launch");
  return KADLLM_OK;
}

}  // namespace
}  // namespace kb

extern "C" int kadllm_gemm(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc,
                           const void* resid, int64_t ld_resid, int64_t M, int64_t N, int64_t K, int64_t n_out,
                           int epilogue, uint32_t* status, void* stream) {
  using namespace kb;
  KB_REQUIRE(a && b && c && status, KADLLM_EINVAL, "gemm: null pointer");
  KB_REQUIRE(M >= 1 && N >= 1 && K >= 1, KADLLM_EINVAL, "gemm: empty dimensions");
  KB_REQUIRE(epilogue >= kStore && epilogue <= kAddResid, KADLLM_EINVAL, "gemm: unknown epilogue %d", epilogue);
  KB_REQUIRE(M < (int64_t(1) << 30) && N < (int64_t(1) << 30) && K < (int64_t(1) << 30), KADLLM_EINVAL,
             "gemm: dimensions too large");
  KB_REQUIRE(lda >= K && ldb >= K && lda % 8 == 0 && ldb % 8 == 0 && ldc % 8 == 0, KADLLM_EINVAL,
             "gemm: leading dimensions must cover K and be multiples of 8 elements");
  KB_REQUIRE(((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(c)) &
              15) == 0,
             KADLLM_EINVAL, "gemm: operands must be 16-byte aligned");
  if (epilogue == kSiluMul) {
    KB_REQUIRE(N % kBN == 0 && n_out >= 1 && n_out <= N / 2, KADLLM_EINVAL,
               "gemm (SiLU-mul): B must hold whole 128-row gate / up block pairs and n_out <= N / 2");
  } else {
    n_out = N;
  }
  KB_REQUIRE(ldc >= n_out, KADLLM_EINVAL, "gemm: ldc shorter than the output row");
  // the tensor-map store writes whole 16-byte granules: a row ending inside one would
  // overwrite the caller's padding past n_out
  KB_REQUIRE(n_out % 8 == 0, KADLLM_EINVAL, "gemm: the output row width %lld is not a multiple of 8",
             static_cast<long long>(n_out));
  if (epilogue == kAddResid) {
    KB_REQUIRE(resid && ld_resid >= N && ld_resid % 8 == 0 && (reinterpret_cast<uintptr_t>(resid) & 15) == 0,
               KADLLM_EINVAL, "gemm (residual): residual pointer / stride invalid");
  }
  KB_REQUIRE((reinterpret_cast<uintptr_t>(c) & 15) == 0 && (epilogue != kAddResid ||
             (reinterpret_cast<uintptr_t>(resid) & 15) == 0), KADLLM_EINVAL, "gemm: outputs must be 16-byte aligned");
  CUtensorMap ma, mb, mc, mr;
  KB_REQUIRE(make_map(&ma, a, M, K, lda, kBM) && make_map(&mb, b, N, K, ldb, kBN / 2) &&
                 make_map(&mc, c, M, n_out, ldc, 32) &&
                 make_map(&mr, epilogue == kAddResid ? resid : c, M, n_out, epilogue == kAddResid ? ld_resid : ldc, 32),
             KADLLM_ECUDA, "gemm: cannot encode the tensor maps (driver entry point cuTensorMapEncodeTiled)");
  GemmArgs g{};
  g.c = static_cast<__nv_bfloat16*>(c);
  g.ldc = ldc;
  g.resid = static_cast<const __nv_bfloat16*>(resid);
  g.ld_resid = ld_resid;
  g.M = int(M);
  g.N = int(N);
  g.K = int(K);
  g.n_out = int(n_out);
  g.tiles_m = int((M + 255) / 256);
  g.tiles_n = int((N + kBN - 1) / kBN);
  g.status = status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (epilogue == kSiluMul) return launch<kSiluMul>(ma, mb, mc, mr, g, s);
  if (epilogue == kAddResid) return launch<kAddResid>(ma, mb, mc, mr, g, s);
  return launch<kStore>(ma, mb, mc, mr, g, s);
}

extern "C" int kadllm_gemm_logits(const void* a, int64_t lda, const void* b, int64_t ldb, void* logits,
                                  int64_t ld_logits, int64_t M, int64_t N, int64_t K, void* workspace,
                                  int64_t workspace_bytes, int64_t batch, int64_t prev_width, uint32_t* status,
                                  void* stream) {
  using namespace kb;
  KB_REQUIRE(a && b && logits && workspace && status, KADLLM_EINVAL, "gemm (logits): null pointer");
  KB_REQUIRE(M >= 1 && N >= 1 && K >= 1 && batch >= 1 && prev_width >= 1 && M == batch * prev_width, KADLLM_EINVAL,
             "gemm (logits): M must be batch * prev_width rows");
  KB_REQUIRE(N <= int64_t(sel::kSumMax) * sel::kChunk && N % 8 == 0, KADLLM_EINVAL,
             "gemm (logits): vocabulary must be a multiple of 8 and at most %d", sel::kSumMax * sel::kChunk);
  KB_REQUIRE(M < (int64_t(1) << 30) && K < (int64_t(1) << 30), KADLLM_EINVAL, "gemm (logits): dimensions too large");
  KB_REQUIRE(lda >= K && ldb >= K && lda % 8 == 0 && ldb % 8 == 0 && ld_logits >= N && ld_logits % 8 == 0,
             KADLLM_EINVAL, "gemm (logits): leading dimensions must cover the rows and be multiples of 8 elements");
  KB_REQUIRE(((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
               reinterpret_cast<uintptr_t>(logits)) & 15) == 0 && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
             KADLLM_EINVAL, "gemm (logits): operands 16-byte aligned, workspace 256-byte aligned");
  const sel::Workspace ws(batch, prev_width);
  KB_REQUIRE(workspace_bytes >= int64_t(ws.fused), KADLLM_EINVAL,
             "gemm (logits): workspace smaller than kadllm_beam_select_workspace_fused");
  CUtensorMap ma, mb, mc;
  KB_REQUIRE(make_map(&ma, a, M, K, lda, kBM) && make_map(&mb, b, N, K, ldb, kBN / 2) &&
                 make_map(&mc, logits, M, N, ld_logits, 32),
             KADLLM_ECUDA, "gemm (logits): cannot encode the tensor maps (driver entry point cuTensorMapEncodeTiled)");
  GemmArgs g{};
  g.c = static_cast<__nv_bfloat16*>(logits);
  g.ldc = ld_logits;
  g.M = int(M);
  g.N = int(N);
  g.K = int(K);
  g.n_out = int(N);
  g.tiles_m = int((M + 255) / 256);
  g.tiles_n = int((N + kBN - 1) / kBN);
  g.status = status;
  char* w = static_cast<char*>(workspace);
  g.vsum = reinterpret_cast<uint16_t*>(w + ws.vsum);
  g.tsum = reinterpret_cast<float*>(w + ws.tsum);
  return launch<kLogits>(ma, mb, mc, mc, g, static_cast<cudaStream_t>(stream));
}
