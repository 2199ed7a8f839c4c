// Persistent warp-specialised BF16 GEMM on the 5th-generation tensor cores.
//
//   D[i, j] = sum_k P[i, k] * Q[j, k]        (both operands K-major, fp32 accumulate)
//
// Normal mode: P = activations A[M, K], Q = weights W[N, K]  -> C[M, N] = A W^T
// Swap-AB mode (small M): P = W, Q = A and the tile is written transposed,
// so the 128-row UMMA M side is filled by weight rows and the token count
// only has to cover the (>= 16) UMMA N side.
//
// Pipeline (one CTA per SM, 6 warps):
//   warp 0      TMA producer: one elected lane streams 128x64 P tiles and
//               BNx64 Q tiles (128-byte swizzle) into a STAGES-deep smem ring.
//   warp 1      TMEM allocator + MMA issuer: one lane issues tcgen05.mma
//               (M=128, N=BN, K=16) into a double-buffered TMEM accumulator and
//               tcgen05.commit's the smem slot back to the producer.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, convert, optional
//               fused SiLU(gate)*up, store bf16 to global. Runs concurrently
//               with the next tile's main loop (accumulator double buffer).
//
// Tall tiles (MH = 2, normal mode only): one CTA owns 256 P rows x BN, as two
// M=128 MMAs per K step that share the Q (weight) tile and write two TMEM
// accumulators. At decode batch sizes (M <= 256) every weight byte then
// enters shared memory once instead of once per 128-row M tile, which cuts
// the L2-to-SM operand traffic by up to a third; the accumulator is double
// buffered while 2 * MH * BN fits the 512 TMEM columns, single buffered above.
//
// Reference parity: replaces the TurboMind sm70 GEMM family
// (sm70/csrc/turbomind/lmdeploy/src/turbomind/kernels/gemm/gemm.h:14-50,
// kernel/sm70_884_*.cu) and its gated-SiLU epilogue (types.h:141); the
// reference computes the same contraction with mma.sync m8n8k4 on sm_70.
//
// Weight-only quantised variants (WF != kWBf16, swap-AB only): the producer
// TMA-loads the raw weight tile (FP8 e4m3 with 128x128 block scales, AWQ int4
// with g128 scale/zero, or NVFP4 e2m1 with e4m3 16-element block scales) into
// a staging buffer; four extra dequant warps convert it to the bf16 128-byte-
// swizzled operand tile (generic-proxy stores + fence.proxy.async) and signal
// the MMA issuer. W8A16 / W4A16 semantics (the reference's TurboMind fp8 /
// awq / nvfp4 ops: sm70/csrc/turbomind/ops/tm_fp8_sm70.cu, tm_awq_sm70.cu,
// tm_nvfp4_sm70.cu).
//
// All mbarrier waits are bounded (common/ptx.cuh); on a timeout every role
// leaves its loop, the MMA issuer drains its outstanding MMAs, the producer
// drains its outstanding TMA copies, and the CTA frees TMEM before exiting.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "common/launch.h"
#include "common/ptx.cuh"
#include "comm/ar_rmsnorm_dev.cuh"
#include "common/tmap.h"
#include "gemm/gemm_api.h"
#include "gemm/dequant.cuh"

namespace b200 {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int UMMA_K = 16;
constexpr int kThreads = 192;    // bf16: producer, MMA, 4 epilogue warps
constexpr int kThreadsQ = 320;   // quantised weights: + 4 dequant warps
constexpr int kGroupM = 16;  // rasterisation group (M tiles) for L2 reuse

struct TileCoord {
  int mb, nb;
};

__device__ __forceinline__ TileCoord tile_coord(int t, int num_m, int num_n) {
  const int per_group = kGroupM * num_n;
  const int g = t / per_group;
  const int first_m = g * kGroupM;
  const int gsize = min(num_m - first_m, kGroupM);
  const int r = t - g * per_group;
  return {first_m + r % gsize, r / gsize};
}

// K-loop start offset per tile when there is a single M tile (decode-sized
// M): tiles running concurrently start at different k-blocks, so the shared
// activation tile is not requested from the same L2 lines by every SM at the
// same moment. With several M tiles the tiles of a wave must walk K in step
// instead (their operands then share L2 lines), so the offset is 0. The
// accumulation order differs per tile but is fixed for a given shape.
__device__ __forceinline__ int kb_rotation(int t, int nk, int num_m) {
  return (nk > 1 && num_m == 1) ? (int)(((unsigned)t * 2654435761u) >> 7) % nk : 0;
}

// Where one tile's operands come from and where its output goes.
struct UnitCoord {
  int p_row, q_row;    // TMA row coordinates of the P / Q operands
  int out_i0, out_j0;  // output index bases along P / Q
  int p_lim, q_lim;    // exclusive bounds for out_i0 + i / out_j0 + j
};

template <int BN>
__device__ __forceinline__ UnitCoord unit_coord(int t, int num_m, int num_n, const GroupInfo& g,
                                                int p_rows, int q_rows, int p_stride = BM) {
  if (g.E > 0) {
    // Grouped (swap-AB): tiles are ordered expert by expert; within an expert,
    // weight-row blocks vary fastest.
    int lo = 0, hi = g.E;  // largest e with tile_off[e] <= t
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (__ldg(g.tile_off + mid) <= t) lo = mid; else hi = mid;
    }
    const int e = lo;
    const int local = t - __ldg(g.tile_off + e);
    const int nbs = g.N / BM;
    const int nb = local % nbs, qb = local / nbs;
    const int r0 = __ldg(g.row_off + e);
    UnitCoord u;
    u.p_row = e * g.N + nb * BM;
    u.q_row = r0 + qb * BN;
    u.out_i0 = nb * BM;
    u.out_j0 = u.q_row;
    u.p_lim = g.N;
    u.q_lim = __ldg(g.row_off + e + 1);
    return u;
  }
  const TileCoord tc = tile_coord(t, num_m, num_n);
  return UnitCoord{tc.mb * p_stride, tc.nb * BN, tc.mb * p_stride, tc.nb * BN, p_rows, q_rows};
}

// Optional per-CTA timeline (profiling aid, off unless a buffer is installed
// with gemm_set_timeline): 16 %globaltimer slots per CTA -- entry, set-up
// done, first TMA issued, first operand stage ready, last MMA issued, first
// accumulator ready, epilogue done, exit, then the split-K epilogue phases
// (partial written, fenced). Buffer layout: kTlCtas launch counters (one per
// block index), then kTlSeqs x kTlCtas rows of 16 stamps. Each CTA takes its
// block's next launch number, so a chain of launches with the same grid
// keeps every launch's stamps (row = launch % kTlSeqs).
__device__ unsigned long long* g_gemm_timeline = nullptr;
constexpr int kSerialSplitFlag = 1 << 16;  // or-ed into the split count
constexpr int kTlCtas = 256;
constexpr int kTlSeqs = 64;

template <int BN, int STAGES, int WF = kWBf16, int MH = 1>
struct Smem {
  static constexpr int kHalfBytes = BM * BK * 2;  // one 128-row P sub-tile
  static constexpr int kPBytes = MH * kHalfBytes;
  static constexpr int kQBytes = BN * BK * 2;
  static constexpr int kRawBytes = BM * raw_row_bytes(WF);  // weight = P side (swap)
  static constexpr int kStageBytes = kPBytes + kQBytes + kRawBytes;
  static constexpr int kTileBytes = STAGES * kStageBytes;
  // Output staging for the tensor-map store: 4 epilogue warps x 2 buffers x
  // (32 rows x 32 bf16) = 16 KB.
  static constexpr int kEpiBytes = 4 * 2 * 32 * 64;
  static constexpr int kBarBytes = 512;
  static constexpr int kTotal = kTileBytes + kEpiBytes + kBarBytes + 1024;  // +1024: alignment
};

template <int BN, int STAGES, bool SWAP, int EPI, int WF = kWBf16, int MH = 1, bool CL = false,
          bool PAIR = false>
__global__ void __launch_bounds__(WF == kWBf16 ? kThreads : kThreadsQ, 1)
gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmap_p,
                    const __grid_constant__ CUtensorMap tmap_q,
                    const __grid_constant__ CUtensorMap tmap_c, __nv_bfloat16* __restrict__ C,
                    int ldc, int p_rows, int q_rows, int K, int splits_arg, float* __restrict__ ws,
                    int* __restrict__ counters, unsigned int* err, const WQParams wq,
                    const GroupInfo grp, const int pm, const int pbox, const int qbox) {
  // Timeline row of this CTA (thread 0 until set-up, then every thread).
  unsigned long long* tl_row = nullptr;
  if (threadIdx.x == 0 && g_gemm_timeline != nullptr && blockIdx.x < kTlCtas) {
    unsigned long long* const tl = g_gemm_timeline;
    const unsigned long long seq = atomicAdd(&tl[blockIdx.x], 1ull) % kTlSeqs;
    tl_row = tl + kTlCtas + (seq * kTlCtas + blockIdx.x) * 16;
  }
  // A negative split count asks for the external reduction (see `ext`);
  // kSerialSplitFlag asks for the serial reduction (see `dist`).
  const bool serial_req = splits_arg > 0 && (splits_arg & kSerialSplitFlag) != 0;
  const int splits = (splits_arg < 0 ? -splits_arg : splits_arg) & (kSerialSplitFlag - 1);
#define B200_TL(i) \
  do { if (tl_row) tl_row[(i)] = globaltimer(); } while (0)
  if (threadIdx.x == 0) B200_TL(0);
  // Programmatic dependent launch: grouped tile lists and quantised
  // operands are read by every role, so those launches wait up front; plain
  // bf16 launches wait in the producer only, after warming L2 with the first
  // weight tiles (weights are never written by an earlier kernel).
  // All-gather -> GEMM (plain normal-mode tiles only; see AgParams).
  constexpr bool kAgKind = EPI == kEpiNone && !SWAP && WF == kWBf16 && !CL && !PAIR;
  const bool ag_on = kAgKind && wq.ag.world > 0;
  const bool early_wait = grp.E > 0 || WF != kWBf16 || ag_on;
  if (early_wait) pdl_wait();
  static_assert(WF == kWBf16 || SWAP, "quantised weights use the swap-AB (weight = P) form");
  static_assert(MH == 1 || (!SWAP && WF == kWBf16), "tall tiles: normal-mode bf16 only");
  static_assert(!CL || (!SWAP && WF == kWBf16), "cluster split-K: normal-mode bf16 only");
  static_assert(!PAIR || (!SWAP && WF == kWBf16 && MH == 1 && !CL), "CTA pair: plain bf16 tiles");
  constexpr bool kQuant = WF != kWBf16;
  constexpr int BMT = BM * MH;  // P rows per tile (per CTA)
  // CTA pair: the tile is 256 P rows x BN; this CTA loads P rows
  // [rank * 128, +128) and Q rows [rank * BN/2, +BN/2) and holds its 128
  // accumulator rows x BN in its own TMEM.
  constexpr int QR = PAIR ? BN / 2 : BN;       // Q rows loaded by this CTA
  constexpr int UT = PAIR ? 2 * BM : BMT;      // P rows per unit tile
  // TMEM columns: the MH accumulators of one tile sit kHalfCols apart; two
  // tiles' accumulators alternate when they fit.
  constexpr int kHalfCols = MH == 1 ? BN : (BN + 31) / 32 * 32;
  constexpr int kAccCols = MH == 1 ? BN : MH * kHalfCols;
  constexpr int kNumAcc = 2 * kAccCols <= 512 ? 2 : 1;
  using S = Smem<QR, STAGES, WF, MH>;
  static_assert((3 * STAGES + 6) * 8 + 40 <= S::kBarBytes, "barrier / slot area");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* const epi_stage = smem + S::kTileBytes;  // [4 warps][2][32 rows x 64 B]
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S::kTileBytes + S::kEpiBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* dq_bar = empty_bar + STAGES;     // [STAGES] dequantised operand ready
  uint64_t* tfull_bar = dq_bar + STAGES;     // [2]
  uint64_t* tempty_bar = tfull_bar + 2;      // [2]
  uint64_t* done_bar = tempty_bar + 2;       // [1]
  uint64_t* recv_bar = done_bar + 1;         // [1] split-K partials landed (bulk path)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);
  unsigned long long** tl_slot = reinterpret_cast<unsigned long long**>(tmem_slot + 4);
  uint64_t* free_bar = reinterpret_cast<uint64_t*>(tmem_slot + 6);  // cluster split: peers idle
  uint32_t* ag_epoch_slot = tmem_slot + 8;  // all-gather: this launch's epoch

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t prank = PAIR ? (cluster_ctarank() & 1u) : 0u;  // rank within the pair
  const bool leader = prank == 0;
  const int unit0 = PAIR ? (int)blockIdx.x / 2 : (int)blockIdx.x;
  const int ustride = PAIR ? (int)gridDim.x / 2 : (int)gridDim.x;
  // P rows per tile: BMT, or fewer (pm, a multiple of 8) for single-half bf16
  // tiles so that the tile count fits the SM count; the MMA still runs
  // M = 128 and the rows past pm (stale shared memory) are never stored.
  const int p_rows_tile = (MH == 1 && !kQuant && grp.E == 0 && pm > 0 && pm < BM) ? pm : BM;
  const int p_tile = PAIR ? UT : (MH == 1 ? p_rows_tile : BMT);  // P-row stride between tiles
  const int num_m = (p_rows + p_tile - 1) / p_tile;
  const int num_n = (q_rows + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;
  const int kb_per = (num_kb + splits - 1) / splits;
  const int num_units = grp.E > 0 ? __ldg(grp.tile_off + grp.E) * splits : num_tiles * splits;
  // Distributed split-K reduction: when every unit runs in the first (only)
  // round, all splits of a tile are resident together, so each split reduces
  // the column chunks it owns (its own partial straight from TMEM, the others'
  // from the workspace) instead of the last-arriving split reducing the whole
  // tile. Same summation order (split 0, 1, ...) as the serial path.
  // External split-K reduction: launched without arrival counters, the
  // splits never meet in this kernel. Each writes its fp32 partial tile into
  // the workspace laid out [split][M][N] (tensor map tmap_c, tile stores
  // staged in the idle operand ring) and the reduction kernel that follows on
  // the stream sums the partials in split order over every SM of the GPU,
  // instead of the split CTAs exchanging them at a handful of loads in flight
  // per thread. One round of units only (the ring must be idle).
  constexpr bool kExtKind = EPI == kEpiNone && !SWAP && WF == kWBf16 && !CL && BN % 32 == 0 &&
                            MH * BN * BM * 4 <= S::kTileBytes;
  // The launcher asks for it only for one round of units and a workspace
  // of splits x M x N floats.
  const bool ext = kExtKind && splits_arg < -1 && ws != nullptr && grp.E == 0 &&
                   num_units <= ustride;
  // Serial instead (requested): the last split to arrive sums the tile; the
  // others leave as soon as their partials are stored, freeing their SMs for
  // the next kernel's CTAs (which start streaming their weights early).
  const bool dist = splits > 1 && grp.E == 0 && num_units <= ustride && !ext && !serial_req;
  // Bulk variant of the distributed reduction (plain epilogue): the partial
  // chunks move between shared memory (the idle operand ring) and the
  // workspace as 16 KB bulk copies instead of per-thread 16-byte accesses, so
  // the exchange runs at copy-engine depth rather than at the few loads each
  // epilogue thread can keep in flight. Needs the staged chunks to fit the ring.
  constexpr int kCW = BN % 32 == 0 ? 32 : 16;
  constexpr int kNCH = BN / kCW;
  constexpr int kChunkBytes = BM * kCW * 4;
  // Largest chunk count any split stages (the chunks it does not own) or
  // receives (the other splits' partials of the chunks it owns); every split
  // of a tile takes the same path.
  const int bulk_stage = splits > 1 ? kNCH - kNCH / splits : 0;
  const int bulk_recv = splits > 1 ? (kNCH + splits - 1) / splits * (splits - 1) : 0;
  const bool bulk = dist && EPI == kEpiNone &&
                    (size_t)MH * kChunkBytes * (bulk_stage > bulk_recv ? bulk_stage : bulk_recv) <=
                        (size_t)S::kTileBytes;
  constexpr int kUsedCols = kNumAcc * kAccCols;
  constexpr uint32_t kTmemCols = (kUsedCols <= 32) ? 32 : (kUsedCols <= 64) ? 64
                                 : (kUsedCols <= 128) ? 128 : (kUsedCols <= 256) ? 256 : 512;
  static_assert(kUsedCols <= 512, "accumulators exceed TMEM");

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
      mbar_init(&dq_bar[s], 4);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], PAIR ? 8 : 4);  // pair: both CTAs' epilogue warps
    }
    mbar_init(done_bar, 1);
    mbar_init(recv_bar, 1);
    mbar_init(free_bar, splits > 1 ? splits - 1 : 1);
    // (all-gather: the previous launch, which bumped the epoch, has completed:
    // early_wait put the PDL wait above)
    *ag_epoch_slot = ag_on ? *(volatile uint32_t*)(wq.ag.pad_local + kAgPadEpoch) + 1u : 0u;
    *abort_flag = 0;
    *tl_slot = tl_row;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_p);
    tma_prefetch_desc(&tmap_q);
  }
  // Plain normal-mode bf16 tiles store through the tensor map: each epilogue
  // warp stages its 32 rows x CW columns in shared memory (64-byte or 32-byte
  // swizzle, matching the map) and one lane issues the tile store, so the
  // global writes go out as whole row segments instead of 16-byte pieces of
  // 32 different rows. Tiles narrower than 128 rows keep the direct stores
  // (their rows past the tile belong to the next tile).
  constexpr bool kTmaStoreKind = EPI == kEpiNone && !SWAP && WF == kWBf16 && !CL;
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  // Pair / cluster split: the peers' TMA completions, bulk copies and barrier
  // arrivals target this CTA's barriers, so every CTA's initialisation must
  // be visible first.
  if constexpr (PAIR || CL) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  tl_row = *tl_slot;
  const uint32_t ag_e = *ag_epoch_slot;
  // Gather-buffer rows of this epoch's half (A tile coordinates are offset by it).
  const int ag_off = ag_on ? (int)(ag_e & 1u) * wq.ag.t_max : 0;
  if (threadIdx.x == 0) {
    B200_TL(1);
    pdl_trigger();
  }
  bool cl_ok = false;  // cluster split: this epilogue thread's accumulator is ready

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // A bulk-tensor instruction costs its warp a few hundred ns, so the L2
    // warm-up and the initial pipeline fill go out lane-parallel (one k-block
    // per lane); the steady-state loop issues from lane 0.
    // parts: bit 0 = P tiles, bit 1 = Q tiles, bit 2 = arm the stage's barrier
    // with the whole stage's bytes (bf16 operands only; quantised stages
    // always load whole).
    auto load_stage = [&](const UnitCoord& uc, int kb, int stage, int parts = 7) {
      uint8_t* spp = smem + stage * S::kStageBytes;
      if constexpr (kQuant) {
        // Activations (Q side, bf16) + the raw weight tile; the P operand is
        // written by the dequant warps.
        mbar_arrive_expect_tx(&full_bar[stage], S::kQBytes + S::kRawBytes);
        tma_load_2d(spp + S::kPBytes, &tmap_q, &full_bar[stage], kb * BK, uc.q_row);
        tma_load_2d(spp + S::kPBytes + S::kQBytes, &tmap_p, &full_bar[stage],
                    kb * raw_row_bytes(WF), uc.p_row);
      } else {
        // Operand tiles go in pbox- / qbox-row TMA boxes (8-row multiples
        // keep the 1024-byte swizzle atoms aligned).
        if constexpr (PAIR) {
          // Both CTAs' halves complete on the leader's barrier, which
          // expects the bytes of the whole pair.
          if (leader && (parts & 4))
            mbar_arrive_expect_tx(&full_bar[stage],
                                  (uint32_t)(2 * (BM * BK * 2 + S::kQBytes)));
          const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0u);
          if (parts & 1)
            for (int r = 0; r < BM; r += pbox)
              tma_load_2d_pair(spp + r * (BK * 2), &tmap_p, fb, kb * BK,
                               uc.p_row + (int)prank * BM + r);
          if (parts & 2)
            for (int r = 0; r < QR; r += qbox)
              tma_load_2d_pair(spp + S::kPBytes + r * (BK * 2), &tmap_q, fb, kb * BK,
                               uc.q_row + (int)prank * QR + r);
        } else {
          if (parts & 4)
            mbar_arrive_expect_tx(&full_bar[stage],
                                  (uint32_t)(MH * p_rows_tile * BK * 2 + S::kQBytes));
          if (parts & 1) {
#pragma unroll
            for (int h = 0; h < MH; ++h)
              for (int r = 0; r < p_rows_tile; r += pbox)
                tma_load_2d(spp + h * S::kHalfBytes + r * (BK * 2), &tmap_p, &full_bar[stage],
                            kb * BK, ag_off + uc.p_row + h * BM + r);
          }
          if (parts & 2)
            for (int r = 0; r < BN; r += qbox)
              tma_load_2d(spp + S::kPBytes + r * (BK * 2), &tmap_q, &full_bar[stage], kb * BK,
                          uc.q_row + r);
        }
      }
    };
    // All-gather: before a unit's first A tile, wait (bounded) until every
    // rank whose rows the tile covers has published them into this rank's
    // gather buffer, then order those peer writes before the tensor-copy reads.
    uint32_t ag_seen = 0;  // ranks already seen ready in this launch
    auto ag_wait = [&](const UnitCoord& uc) -> bool {
      if (!ag_on) return true;
      const int rpr = wq.ag.rows_per_rank;
      const int r0 = uc.p_row, r1 = min(p_rows, uc.p_row + MH * BM) - 1;
      if (r1 < r0) return true;
      const int c0 = r0 / rpr, c1 = min(wq.ag.world - 1, r1 / rpr);
      for (int c = c0; c <= c1; ++c) {
        if ((ag_seen >> c) & 1u) continue;
        if (!ardev::wait_geq(wq.ag.pad_local + kAgPadReady + c, ag_e, err, wq.ag.timeout_ns))
          return false;
        ag_seen |= 1u << c;
      }
      fence_proxy_async_global();
      return true;
    };
    int pre = 0;  // k-blocks of the first unit issued lane-parallel
    if (unit0 < num_units) {
      const int t = unit0 / splits, sp = unit0 - t * splits;
      const UnitCoord uc = unit_coord<BN>(t, num_m, num_n, grp, p_rows, q_rows, p_tile);
      const int kb0 = sp * kb_per, kb1 = min(num_kb, kb0 + kb_per);
      const int nk = kb1 - kb0;
      const int rot = kb_rotation(t, nk, num_m);
      if constexpr (!kQuant) pre = max(0, min(nk, STAGES));
      if (!early_wait) {
        // Before waiting for the previous kernel (weights are never written
        // by an earlier kernel): issue the weight tiles of the first-round
        // stages straight into the ring, each stage's barrier armed with the
        // whole stage's bytes, and pull the weights of the next STAGES
        // k-blocks into L2. Only the activation tiles wait for the previous
        // kernel's results.
        constexpr int kW = SWAP ? 1 : 2, kA = SWAP ? 2 : 1;
        for (int it = pre + lane; it < min(nk, 2 * STAGES); it += 32) {
          const int kb = kb0 + (it + rot) % nk;
          if constexpr (SWAP) {
            for (int r = 0; r < p_rows_tile; r += pbox)
              tma_prefetch_l2_2d(&tmap_p, kb * BK, uc.p_row + r);
          } else {
            for (int r = 0; r < QR; r += qbox)
              tma_prefetch_l2_2d(&tmap_q, kb * BK, uc.q_row + (int)prank * QR + r);
          }
        }
        if (lane < pre) load_stage(uc, kb0 + (lane + rot) % nk, lane, 4 | kW);
        if (lane == 0 && pre > 0) B200_TL(2);
        pdl_wait();
        if (lane < pre) load_stage(uc, kb0 + (lane + rot) % nk, lane, kA);
      } else if constexpr (!kQuant) {
        if (!ag_wait(uc)) {
          *abort_flag = 1;
          pre = 0;
        }
        if (lane < pre) load_stage(uc, kb0 + (lane + rot) % nk, lane);
        if (lane == 0 && pre > 0) B200_TL(2);
      }
    }
    __syncwarp();
    if (lane == 0) {
      int stage = pre % STAGES;
      uint32_t phase = pre == STAGES ? 1u : 0u;
      long issued = pre;
      bool first = true;
      for (int u = unit0; u < num_units && !*abort_flag; u += ustride) {
        const int t = u / splits, sp = u - t * splits;
        const UnitCoord uc = unit_coord<BN>(t, num_m, num_n, grp, p_rows, q_rows, p_tile);
        const int kb0 = sp * kb_per, kb1 = min(num_kb, kb0 + kb_per);
        const int nk = kb1 - kb0;
        const int rot = kb_rotation(t, nk, num_m);
        if (!first && !ag_wait(uc)) {
          *abort_flag = 1;
          break;
        }
        for (int it = first ? pre : 0; it < nk; ++it) {
          const int kb = kb0 + (it + rot) % nk;
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, err)) {
            *abort_flag = 1;
            break;
          }
          load_stage(uc, kb, stage);
          if (issued == 0) B200_TL(2);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        first = false;
      }
      // Drain: wait for the copies this warp issued into each slot (bounded).
      // A pair's second CTA counts its copies on the leader's barriers; its
      // operands are consumed (and so landed) before the leader's final
      // commit, which this CTA waits for before tearing down.
      const long n_drain = (PAIR && !leader) ? 0 : (issued < STAGES ? issued : STAGES);
      for (long j = 0; j < n_drain; ++j) {
        const long it = issued - 1 - j;
        mbar_wait(&full_bar[it % STAGES], (uint32_t)((it / STAGES) & 1), err);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && PAIR && !leader) {
      // The leader issues the pair's MMAs; its final commit lands here too.
      mbar_wait(done_bar, 0, err);
    } else if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(PAIR ? 2 * BM : BM, BN, true);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int u = unit0; u < num_units && !*abort_flag; u += ustride, ++local) {
        const int t = u / splits, sp = u - t * splits;
        (void)t;
        const int kb0 = sp * kb_per, kb1 = min(num_kb, kb0 + kb_per);
        const int acc = kNumAcc == 2 ? (local & 1) : 0;
        const uint32_t acc_phase = kNumAcc == 2 ? ((local >> 1) & 1) : (local & 1);
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, err)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kAccCols;
        bool ok = true;
        for (int it = 0; it < kb1 - kb0; ++it) {
          if (!mbar_wait(kQuant ? &dq_bar[stage] : &full_bar[stage], phase, err)) {
            ok = false;
            break;
          }
          if (local == 0 && it == 0) B200_TL(3);
          tc_fence_after();
          const uint32_t spa = smem_u32(smem + stage * S::kStageBytes);
          const uint64_t bdesc = umma_desc_sw128(spa + S::kPBytes);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            // +32 bytes per K=16 step inside the 128-byte swizzle row.
#pragma unroll
            for (int h = 0; h < MH; ++h) {
              const uint64_t adesc = umma_desc_sw128(spa + h * S::kHalfBytes);
              if constexpr (PAIR) {
                umma_f16_pair(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                              (it > 0 || k > 0) ? 1u : 0u);
              } else {
                umma_f16(d_tmem + h * kHalfCols, adesc + (uint64_t)(2 * k),
                         bdesc + (uint64_t)(2 * k), idesc, (it > 0 || k > 0) ? 1u : 0u);
              }
            }
          }
          if constexpr (PAIR) umma_commit_pair(&empty_bar[stage], 0x3);
          else umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if constexpr (PAIR) umma_commit_pair(&tfull_bar[acc], 0x3);
        else umma_commit(&tfull_bar[acc]);
        if (!ok) {
          *abort_flag = 1;
          break;
        }
      }
      B200_TL(4);
      // Make sure no MMA is still writing TMEM before it is freed.
      if constexpr (PAIR) umma_commit_pair(done_bar, 0x3);
      else umma_commit(done_bar);
      mbar_wait(done_bar, 0, err);
    }
    __syncwarp();
  } else if (kQuant && warp >= 6) {
    // ------------------------------------------------------------ dequant warps
    const int dt = threadIdx.x - 192;  // 0..127
    const int c = dt & 7;              // 16-byte chunk (8 k) of the row
    int stage = 0;
    uint32_t phase = 0;
    for (int u = unit0; u < num_units && !*abort_flag; u += ustride) {
      const int t = u / splits, sp = u - t * splits;
      const UnitCoord uc = unit_coord<BN>(t, num_m, num_n, grp, p_rows, q_rows);
      const int kb0 = sp * kb_per, kb1 = min(num_kb, kb0 + kb_per);
      const int nk = kb1 - kb0;
      const int rot = kb_rotation(t, nk, num_m);
      for (int it = 0; it < nk; ++it) {
        const int kb = kb0 + (it + rot) % nk;
        // The 8 rows' scales do not depend on the TMA copy: issue their loads
        // first so that their latency overlaps the wait for the weight bytes.
        typename DqScale<WF>::type sc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int n = uc.p_row + (dt >> 3) + 16 * j;
          sc[j] = dq_scale<WF>(wq, n < p_rows ? n : 0, kb, c);
        }
        if (!mbar_wait(&full_bar[stage], phase, err)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* spp = smem + stage * S::kStageBytes;
        const uint8_t* raw = spp + S::kPBytes + S::kQBytes;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int r = (dt >> 3) + 16 * j;  // tile row 0..127
          const int n = uc.p_row + r;        // weight row (stacked for grouped)
          uint4 v = make_uint4(0, 0, 0, 0);
          if (n < p_rows) v = dequant8_s<WF>(raw + r * raw_row_bytes(WF), c, sc[j]);
          *reinterpret_cast<uint4*>(spp + r * 128 + ((c ^ (r & 7)) << 4)) = v;
        }
        // Generic-proxy smem writes -> visible to the tensor core (async proxy).
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if ((dt & 31) == 0) mbar_arrive(&dq_bar[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if constexpr (CL) {
    // ------------------------------------------------------------ epilogue (cluster split)
    // One unit per CTA: wait for the accumulator; the exchange and the
    // reduction run after the role branches, where every thread of the
    // cluster can join the cluster barriers.
    if ((int)blockIdx.x < num_units && !*abort_flag) {
      cl_ok = mbar_wait(&tfull_bar[0], 0, err);
      if (!cl_ok) *abort_flag = 1;
      else tc_fence_after();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = q * 32 + lane;
    const int etid = threadIdx.x - 64;  // 0..127
    constexpr int CW = BN % 32 == 0 ? 32 : 16;  // columns per tcgen05.ld
    static_assert(BN % CW == 0, "tile width must be a multiple of 16");
    const float out_scale = wq.out_scale;
    const bool tma_st = kTmaStoreKind && (PAIR || MH == 2 || p_rows_tile == BM);
    int ebuf = 0;  // staging buffer of this warp's next tile store
    if (ag_on) {
      // All-gather: copy this rank's rows into slot `rank` of this epoch's half
      // of every rank's gather buffer (16-byte stores over NVLink), while the
      // producer and the tensor core start on the rows already here. The last
      // CTA to finish publishes the rank's ready flag on every rank.
      const AgParams& ag = wq.ag;
      const size_t nvec = (size_t)ag.rows_per_rank * ag.K / 8;
      const size_t dst0 = ((size_t)(ag_e & 1u) * ag.t_max + (size_t)ag.rank * ag.rows_per_rank) *
                          ag.K / 8;
      const uint4* src = reinterpret_cast<const uint4*>(ag.shard);
      for (size_t i = (size_t)blockIdx.x * 128 + etid; i < nvec; i += (size_t)gridDim.x * 128) {
        const uint4 v = src[i];
        for (int q2 = 0; q2 < ag.world; ++q2)
          reinterpret_cast<uint4*>(ag.xfull_peer[q2])[dst0 + i] = v;
      }
      __threadfence_system();
      named_barrier_sync(1, 128);
      if (etid == 0) {
        const uint32_t n = atomicAdd(ag.pad_local + kAgPadArrive, 1u) + 1u;
        if (n == gridDim.x) {
          atomicExch(ag.pad_local + kAgPadArrive, 0u);  // re-arm for the next launch
          __threadfence_system();
          for (int q2 = 0; q2 < ag.world; ++q2)
            ardev::st_release_sys(ag.pad_peer[q2] + kAgPadReady + ag.rank, ag_e);
        }
      }
    }
    int local = 0;
    for (int u = unit0; u < num_units && !*abort_flag; u += ustride, ++local) {
      const int t = u / splits, sp = u - t * splits;
      const UnitCoord uc = unit_coord<BN>(t, num_m, num_n, grp, p_rows, q_rows, p_tile);
      const int acc = kNumAcc == 2 ? (local & 1) : 0;
      const uint32_t acc_phase = kNumAcc == 2 ? ((local >> 1) & 1) : (local & 1);
      if (!mbar_wait(&tfull_bar[acc], acc_phase, err)) {
        *abort_flag = 1;
        break;
      }
      if (local == 0 && threadIdx.x == 64) B200_TL(5);
      tc_fence_after();
      const uint32_t t_acc = tmem_base + ((uint32_t)(q * 32) << 16) + acc * kAccCols;
      const bool split = splits > 1;
      // Tile-local fp32 partials of this unit: ws[(t * splits + s)][h][col][row]
      // (a pair's CTAs own halves h = 0 / 1 and count arrivals separately).
      float* ws_tile = split ? ws + (size_t)t * splits * (UT * BN) : nullptr;
      const int hbase = PAIR ? (int)prank : 0;
      // Release this accumulator buffer: a pair's MMA issuer sits in the leader.
      auto release_acc = [&]() {
        if constexpr (PAIR) {
          if (leader) mbar_arrive(&tempty_bar[acc]);
          else mbar_arrive_cluster(mapa_shared(smem_u32(&tempty_bar[acc]), 0u));
        } else {
          mbar_arrive(&tempty_bar[acc]);
        }
      };

      // Ownership of column chunks in the distributed reduction: CW-wide
      // chunks (whole 128-column gate/up blocks for the SiLU epilogue) are
      // dealt round-robin to the splits.
      auto owned = [&](int col0) -> bool {
        if (!dist) return true;
        const int unit = EPI == kEpiSiluMul ? col0 / 128 : col0 / CW;
        return unit % splits == sp;
      };
      const int ci = PAIR ? 2 * t + (int)prank : t;  // arrival counter of this tile (half)
      // Bulk path: chunk ch is owned by split ch % splits; this split owns
      // chunks sp, sp + splits, ...; received partials of owned chunk ch from
      // split s2 sit in ring slot ((h * n_own + ch / splits) * (splits - 1) + s2'),
      // s2' = s2 minus one past this split.
      const int n_own = (kNCH - sp + splits - 1) / splits;
      if (ext) {
        // Stage this warp's 32 rows of every 32-column chunk (fp32, 128-byte
        // swizzle as the map expects), hand the accumulator back, then one
        // lane per chunk issues its tile store (one warp-wide instruction).
        constexpr int kChunks = MH * (BN / 32);
        uint8_t* wst = smem + (size_t)q * kChunks * 4096;
        // Two 32-column TMEM loads per wait: the load latency, not the bytes,
        // bounds this loop.
        auto stage_chunk = [&](int c, const uint32_t (&r)[32]) {
          float4* dst = reinterpret_cast<float4*>(wst + (size_t)c * 4096) + lane * 8;
#pragma unroll
          for (int v = 0; v < 8; ++v)
            dst[v ^ (lane & 7)] =
                make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                            __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
        };
#pragma unroll 1
        for (int h = 0; h < MH; ++h) {
#pragma unroll 1
          for (int ch = 0; ch < BN / 32; ch += 2) {
            uint32_t r0[32], r1[32];
            tmem_ld_32x32b_x32(t_acc + h * kHalfCols + ch * 32, r0);
            if (ch + 1 < BN / 32) tmem_ld_32x32b_x32(t_acc + h * kHalfCols + (ch + 1) * 32, r1);
            tmem_wait_ld();
            stage_chunk(h * (BN / 32) + ch, r0);
            if (ch + 1 < BN / 32) stage_chunk(h * (BN / 32) + ch + 1, r1);
          }
        }
        fence_proxy_async_shared();
        tc_fence_before();
        __syncwarp();
        if (etid == 0) B200_TL(10);
        if (lane == 0) release_acc();
        if (lane < kChunks) {
          const int h = lane / (BN / 32), ch = lane % (BN / 32);
          tma_store_3d(&tmap_c, wst + (size_t)lane * 4096, uc.out_j0 + ch * 32,
                       uc.out_i0 + (hbase + h) * BM + q * 32, sp);
          bulk_commit();
          bulk_wait_all();
        }
        __syncwarp();
        if (etid == 0) B200_TL(11);
        continue;
      }
      if (split && bulk) {
        // Phase A: stage the chunks other splits own (rows swizzled by float4
        // to spread shared-memory banks; the reader uses the same rule).
        int slot = 0;
#pragma unroll 1
        for (int h = 0; h < MH; ++h) {
          const uint32_t t_row = t_acc + h * kHalfCols;
#pragma unroll 1
          for (int ch = 0; ch < kNCH; ++ch) {
            if (ch % splits == sp) continue;
            uint32_t r[32];
            if constexpr (kCW == 32) {
              tmem_ld_32x32b_x32(t_row + ch * kCW, r);
            } else {
              tmem_ld_32x32b_x16(t_row + ch * kCW, *reinterpret_cast<uint32_t(*)[16]>(r));
            }
            tmem_wait_ld();
            float4* dst = reinterpret_cast<float4*>(smem + (size_t)slot * kChunkBytes) +
                          row_in_tile * (kCW / 4);
#pragma unroll
            for (int v = 0; v < kCW / 4; ++v)
              dst[v ^ (row_in_tile & (kCW / 4 - 1))] =
                  make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                              __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
            ++slot;
          }
        }
        fence_proxy_async_shared();
        named_barrier_sync(1, 128);
        if (etid == 0) {
          B200_TL(10);
          // Phase B: one thread copies the staged chunks out, publishes this
          // split's arrival and waits for the others'.
          slot = 0;
          for (int h = 0; h < MH; ++h)
            for (int ch = 0; ch < kNCH; ++ch) {
              if (ch % splits == sp) continue;
              bulk_store(ws_tile + (size_t)sp * (UT * BN) + (size_t)(hbase + h) * (BM * BN) +
                             (size_t)ch * (BM * kCW),
                         smem + (size_t)slot * kChunkBytes, kChunkBytes);
              ++slot;
            }
          bulk_commit();
          bulk_wait_all();
          B200_TL(11);
          fence_proxy_async_global();
          __threadfence();
          atomicAdd(&counters[ci], 1);
          const bool ok = wait_geq_gpu(&counters[ci], splits, err);
          B200_TL(12);
          if (ok) {
            // Phase C: fetch the other splits' partials of the owned chunks.
            fence_proxy_async_global();
            mbar_arrive_expect_tx(recv_bar,
                                  (uint32_t)(MH * n_own * (splits - 1) * kChunkBytes));
            slot = 0;
            for (int h = 0; h < MH; ++h)
              for (int ch = sp; ch < kNCH; ch += splits)
                for (int s2 = 0; s2 < splits; ++s2) {
                  if (s2 == sp) continue;
                  bulk_load(smem + (size_t)slot * kChunkBytes,
                            ws_tile + (size_t)s2 * (UT * BN) + (size_t)(hbase + h) * (BM * BN) +
                                (size_t)ch * (BM * kCW),
                            kChunkBytes, recv_bar);
                  ++slot;
                }
          }
          *last_flag = ok ? 1 : 0;
        }
        named_barrier_sync(1, 128);
        const int arrived = *last_flag;
        named_barrier_sync(1, 128);  // last_flag is rewritten below
        const bool landed = arrived && mbar_wait(recv_bar, 0, err);
        if (etid == 0) B200_TL(13);
        if (!landed) {
          *abort_flag = 1;
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release_acc();
          break;
        }
      } else if (split && dist) {
        // Publish the chunks the other splits own (same workspace layout as
        // the serial path), then wait until every split of the tile has.
#pragma unroll 1
        for (int h = 0; h < MH; ++h) {
          float4* mine = reinterpret_cast<float4*>(ws_tile + (size_t)sp * (UT * BN) +
                                                   (size_t)(hbase + h) * (BM * BN)) +
                         row_in_tile;
          const uint32_t t_row = t_acc + h * kHalfCols;
#pragma unroll 1
          for (int ch = 0; ch < BN / CW; ++ch) {
            if (owned(ch * CW)) continue;
            uint32_t r[32];
            if constexpr (CW == 32) {
              tmem_ld_32x32b_x32(t_row + ch * CW, r);
            } else {
              tmem_ld_32x32b_x16(t_row + ch * CW, *reinterpret_cast<uint32_t(*)[16]>(r));
            }
            tmem_wait_ld();
#pragma unroll
            for (int v = 0; v < CW / 4; ++v)
              __stcg(mine + (size_t)(ch * (CW / 4) + v) * BM,
                     make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                 __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3])));
          }
        }
        __threadfence();
        named_barrier_sync(1, 128);
        if (etid == 0) {
          atomicAdd(&counters[ci], 1);
          *last_flag = wait_geq_gpu(&counters[ci], splits, err) ? 1 : 0;
        }
        named_barrier_sync(1, 128);
        const int arrived = *last_flag;
        named_barrier_sync(1, 128);  // last_flag is rewritten below
        if (!arrived) {
          *abort_flag = 1;
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release_acc();
          break;
        }
        __threadfence();
      }
      if (split && !dist) {
        // Column-group-major layout [BN/4][BM] of float4 per M half: the 32
        // lanes of a warp (consecutive rows) write 512 contiguous bytes per store.
#pragma unroll 1
        for (int h = 0; h < MH; ++h) {
          float4* mine = reinterpret_cast<float4*>(ws_tile + (size_t)sp * (UT * BN) +
                                                   (size_t)(hbase + h) * (BM * BN)) +
                         row_in_tile;
          const uint32_t t_row = t_acc + h * kHalfCols;
#pragma unroll 1
          for (int ch = 0; ch < BN / CW; ++ch) {
            uint32_t r[32];
            if constexpr (CW == 32) {
              tmem_ld_32x32b_x32(t_row + ch * CW, r);
            } else {
              tmem_ld_32x32b_x16(t_row + ch * CW, *reinterpret_cast<uint32_t(*)[16]>(r));
            }
            tmem_wait_ld();
#pragma unroll
            for (int v = 0; v < CW / 4; ++v)
              __stcg(mine + (size_t)(ch * (CW / 4) + v) * BM,
                     make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                 __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3])));
          }
        }
        // The accumulator is in global memory now: release TMEM early.
        if (etid == 0) B200_TL(8);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release_acc();
        __threadfence();
        if (etid == 0) B200_TL(9);
        named_barrier_sync(1, 128);
        if (etid == 0) {
          const int old = atomicAdd(&counters[ci], 1);
          const int last = old == splits - 1;
          if (last) counters[ci] = 0;  // re-arm for the next launch
          *last_flag = last;
        }
        named_barrier_sync(1, 128);
        const int is_last = *last_flag;
        named_barrier_sync(1, 128);  // last_flag may be rewritten by the next unit
        if (!is_last) continue;
        __threadfence();
      }

#pragma unroll 1
      for (int h = 0; h < MH; ++h) {
      const uint32_t t_row = t_acc + h * kHalfCols;
      const int i = uc.out_i0 + (hbase + h) * BM + row_in_tile;  // output index along P
      const bool row_ok = row_in_tile < p_rows_tile;
      const float* ws_half = split ? ws_tile + (size_t)(hbase + h) * (BM * BN) : nullptr;
      // Fetch 32 (or 16) tile columns of this thread's row: from TMEM, or the
      // fixed-order (split 0, 1, ...) sum of the partials.
      auto fetch = [&](int col0, float (&v)[32]) {
        if (bulk) {
          uint32_t r[32];
          if constexpr (CW == 32) {
            tmem_ld_32x32b_x32(t_row + col0, r);
          } else {
            tmem_ld_32x32b_x16(t_row + col0, *reinterpret_cast<uint32_t(*)[16]>(r));
          }
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < CW; ++c) v[c] = 0.f;
          const int base = (h * n_own + (col0 / CW) / splits) * (splits - 1);
          for (int s2 = 0; s2 < splits; ++s2) {
            if (s2 == sp) {
#pragma unroll
              for (int c = 0; c < CW; ++c) v[c] += __uint_as_float(r[c]);
            } else {
              const float4* src =
                  reinterpret_cast<const float4*>(
                      smem + (size_t)(base + (s2 < sp ? s2 : s2 - 1)) * kChunkBytes) +
                  row_in_tile * (CW / 4);
#pragma unroll
              for (int c4 = 0; c4 < CW / 4; ++c4) {
                const float4 x = src[c4 ^ (row_in_tile & (CW / 4 - 1))];
                v[4 * c4] += x.x;
                v[4 * c4 + 1] += x.y;
                v[4 * c4 + 2] += x.z;
                v[4 * c4 + 3] += x.w;
              }
            }
          }
#pragma unroll
          for (int c = 0; c < CW; ++c) v[c] *= out_scale;
        } else if (dist) {
          uint32_t r[32];
          if constexpr (CW == 32) {
            tmem_ld_32x32b_x32(t_row + col0, r);
          } else {
            tmem_ld_32x32b_x16(t_row + col0, *reinterpret_cast<uint32_t(*)[16]>(r));
          }
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < CW; ++c) v[c] = 0.f;
          for (int s2 = 0; s2 < splits; ++s2) {
            if (s2 == sp) {
#pragma unroll
              for (int c = 0; c < CW; ++c) v[c] += __uint_as_float(r[c]);
            } else {
              const float4* src =
                  reinterpret_cast<const float4*>(ws_half + (size_t)s2 * (UT * BN)) +
                  (size_t)(col0 / 4) * BM + row_in_tile;
              float4 x[CW / 4];
#pragma unroll
              for (int c4 = 0; c4 < CW / 4; ++c4) x[c4] = __ldcg(src + (size_t)c4 * BM);
#pragma unroll
              for (int c4 = 0; c4 < CW / 4; ++c4) {
                v[4 * c4] += x[c4].x;
                v[4 * c4 + 1] += x[c4].y;
                v[4 * c4 + 2] += x[c4].z;
                v[4 * c4 + 3] += x[c4].w;
              }
            }
          }
#pragma unroll
          for (int c = 0; c < CW; ++c) v[c] *= out_scale;
        } else if (!split) {
          uint32_t r[32];
          if constexpr (CW == 32) {
            tmem_ld_32x32b_x32(t_row + col0, r);
          } else {
            tmem_ld_32x32b_x16(t_row + col0, *reinterpret_cast<uint32_t(*)[16]>(r));
          }
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < CW; ++c) v[c] = __uint_as_float(r[c]) * out_scale;
        } else {
#pragma unroll
          for (int c = 0; c < CW; ++c) v[c] = 0.f;
          // Up to 4 splits' partials are requested before any is consumed, so a
          // chunk costs one L2 round trip per 4 splits; the adds stay in split
          // order (deterministic).
          constexpr int RG = EPI == kEpiSiluMul ? 2 : 4;  // splits per load batch
          for (int s0 = 0; s0 < splits; s0 += RG) {
            float4 x[RG][CW / 4];
#pragma unroll
            for (int j = 0; j < RG; ++j) {
              if (s0 + j < splits) {
                const float4* src =
                    reinterpret_cast<const float4*>(ws_half + (size_t)(s0 + j) * (UT * BN)) +
                    (size_t)(col0 / 4) * BM + row_in_tile;
#pragma unroll
                for (int c4 = 0; c4 < CW / 4; ++c4) x[j][c4] = __ldcg(src + (size_t)c4 * BM);
              }
            }
#pragma unroll
            for (int j = 0; j < RG; ++j) {
              if (s0 + j < splits) {
#pragma unroll
                for (int c4 = 0; c4 < CW / 4; ++c4) {
                  v[4 * c4] += x[j][c4].x;
                  v[4 * c4 + 1] += x[j][c4].y;
                  v[4 * c4 + 2] += x[j][c4].z;
                  v[4 * c4 + 3] += x[j][c4].w;
                }
              }
            }
          }
#pragma unroll
          for (int c = 0; c < CW; ++c) v[c] *= out_scale;
        }
      };

      if constexpr (EPI == kEpiSiluMul) {
        // Tile columns hold [gate 64 | up 64] blocks; output has BN/2 columns.
#pragma unroll 1
        for (int blk = 0; blk < BN / 128; ++blk) {
#pragma unroll 1
          for (int half = 0; half < 2; ++half) {
            if (!owned(blk * 128)) continue;
            float g[32], uu[32];
            fetch(blk * 128 + half * 32, g);
            fetch(blk * 128 + 64 + half * 32, uu);
            const int j0 = (uc.q_row / BN) * (BN / 2) + blk * 64 + half * 32;
            if (row_ok && i < uc.p_lim) {
              uint32_t packed[16];
#pragma unroll
              for (int c = 0; c < 16; ++c) {
                const float g0 = g[2 * c], g1 = g[2 * c + 1];
                const float o0 = __fdividef(g0, 1.0f + __expf(-g0)) * uu[2 * c];
                const float o1 = __fdividef(g1, 1.0f + __expf(-g1)) * uu[2 * c + 1];
                packed[c] = pack_bf16x2(o0, o1);
              }
              __nv_bfloat16* dst = C + (size_t)i * ldc + j0;
              const int out_cols = q_rows / 2;
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                if (j0 + v * 8 + 8 <= out_cols)
                  *reinterpret_cast<uint4*>(dst + v * 8) =
                      make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2],
                                 packed[4 * v + 3]);
              }
            }
          }
        }
      } else {
#pragma unroll 1
        for (int ch = 0; ch < BN / CW; ++ch) {
          if (!owned(ch * CW)) continue;
          float r[32];
          fetch(ch * CW, r);
          const int j0 = uc.out_j0 + ch * CW;
          if constexpr (kTmaStoreKind) {
            if (tma_st) {
              uint8_t* buf = epi_stage + (size_t)(q * 2 + ebuf) * 2048;
              if (lane == 0) bulk_wait_read_le1();  // this buffer's previous store has read it
              __syncwarp();
#pragma unroll
              for (int v = 0; v < CW / 8; ++v) {
                uint4 pk;
                pk.x = pack_bf16x2(r[8 * v + 0], r[8 * v + 1]);
                pk.y = pack_bf16x2(r[8 * v + 2], r[8 * v + 3]);
                pk.z = pack_bf16x2(r[8 * v + 4], r[8 * v + 5]);
                pk.w = pack_bf16x2(r[8 * v + 6], r[8 * v + 7]);
                // 16-byte unit v of row `lane`: 64-byte rows use the 64B
                // swizzle (unit ^= (row >> 1) & 3), 32-byte rows the 32B one.
                const int u = CW == 32 ? (v ^ ((lane >> 1) & 3)) : (v ^ ((lane >> 2) & 1));
                *reinterpret_cast<uint4*>(buf + lane * (CW * 2) + u * 16) = pk;
              }
              fence_proxy_async_shared();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&tmap_c, buf, j0, i - lane);
                bulk_commit();
              }
              ebuf ^= 1;
              continue;
            }
          }
          if constexpr (!SWAP) {
            if (row_ok && i < uc.p_lim) {
              __nv_bfloat16* dst = C + (size_t)i * ldc + j0;
#pragma unroll
              for (int v = 0; v < CW / 8; ++v) {
                if (j0 + v * 8 + 8 <= uc.q_lim) {
                  uint4 pk;
                  pk.x = pack_bf16x2(r[8 * v + 0], r[8 * v + 1]);
                  pk.y = pack_bf16x2(r[8 * v + 2], r[8 * v + 3]);
                  pk.z = pack_bf16x2(r[8 * v + 4], r[8 * v + 5]);
                  pk.w = pack_bf16x2(r[8 * v + 6], r[8 * v + 7]);
                  *reinterpret_cast<uint4*>(dst + v * 8) = pk;
                }
              }
            }
          } else {
            // Transposed store: lane i holds P row i (an output column);
            // consecutive lanes write consecutive bf16 of one output row.
            if (row_ok && i < uc.p_lim) {
#pragma unroll
              for (int c = 0; c < CW; ++c) {
                const int j = j0 + c;
                if (j < uc.q_lim) C[(size_t)j * ldc + i] = __float2bfloat16_rn(r[c]);
              }
            }
          }
        }
      }
      }  // M halves
      if (!split || dist) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release_acc();
      }
      if (dist) {
        // Every split of the tile has passed its wait once the counter reaches
        // 2 x splits; the last one re-arms it for the next launch.
        named_barrier_sync(1, 128);
        if (etid == 0) {
          const int old = atomicAdd(&counters[ci], 1);
          if (old == 2 * splits - 1) counters[ci] = 0;
        }
      }
    }
    // The staged tiles must be read out before shared memory goes away.
    if (tma_st && lane == 0) bulk_wait_all();
  }

  // Cluster split-K by bulk copies (plain epilogue, 128-row tiles): the tile's
  // 32-column chunks are dealt round-robin to the splits (chunk ch belongs to
  // split ch % splits, the cluster rank). Each CTA stages the chunks it does
  // not own in its idle operand ring, grouped by owner; tells every peer that
  // its own ring is idle and its receive barrier armed (remote arrive); once
  // all peers have said so, one thread copies each owner's group into that
  // owner's receive area with a single shared::cta -> shared::cluster bulk
  // copy. Every CTA then sums its owned chunks over the splits in split order
  // (its own partial straight from TMEM) and stores bf16 tiles through the
  // output tensor map. Ring use per CTA: the staged chunks, then the received
  // ones: (chunks - owned) + (splits - 1) x owned chunks of 16 KB.
  constexpr bool kClBulkKind = CL && EPI == kEpiNone && MH == 1 && BN % 32 == 0;
  constexpr int kClChunks = BN / 32;
  constexpr int kClChunkBytes = BM * 32 * 4;
  const int cl_need = kClChunks - kClChunks / (splits > 0 ? splits : 1) +
                      (splits - 1) * ((kClChunks + splits - 1) / (splits > 0 ? splits : 1));
  const bool cl_bulk = kClBulkKind && splits > 1 &&
                       (size_t)cl_need * kClChunkBytes <= (size_t)S::kTileBytes;
  if constexpr (kClBulkKind) {
  if (cl_bulk && warp >= 2) {
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    const int etid = threadIdx.x - 64;
    const int sp = (int)cluster_ctarank();
    const int ns = splits;
    const int t = (int)blockIdx.x / ns;
    const UnitCoord uc = unit_coord<BN>(t, num_m, num_n, grp, p_rows, q_rows, p_tile);
    const uint32_t t_acc = tmem_base + ((uint32_t)(q * 32) << 16);
    auto n_own_of = [&](int d) { return (kClChunks - d + ns - 1) / ns; };
    const int my_own = n_own_of(sp);
    // Receive area of CTA d: right after its staged chunks, [source][owned chunk].
    auto recv_chunk = [&](int d, int src_slot, int k) {
      return (kClChunks - n_own_of(d)) + src_slot * n_own_of(d) + k;
    };
    auto put = [&](int slot, const uint32_t (&r)[32]) {
      float4* dst = reinterpret_cast<float4*>(smem + (size_t)slot * kClChunkBytes) +
                    row_in_tile * 8;
#pragma unroll
      for (int v = 0; v < 8; ++v)
        dst[v ^ (row_in_tile & 7)] =
            make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                        __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
    };
    if (cl_ok) {
      // Stage the chunks the other splits own, grouped by owner (two TMEM
      // loads in flight per wait).
      int slot = 0;
#pragma unroll 1
      for (int d = 0; d < ns; ++d) {
        if (d == sp) continue;
#pragma unroll 1
        for (int ch = d; ch < kClChunks; ch += 2 * ns) {
          uint32_t r0[32], r1[32];
          const bool two = ch + ns < kClChunks;
          tmem_ld_32x32b_x32(t_acc + ch * 32, r0);
          if (two) tmem_ld_32x32b_x32(t_acc + (ch + ns) * 32, r1);
          tmem_wait_ld();
          put(slot++, r0);
          if (two) put(slot++, r1);
        }
      }
    }
    fence_proxy_async_shared();
    named_barrier_sync(1, 128);
    if (etid == 0) {
      bool ok = cl_ok;
      if (ok) {
        mbar_arrive_expect_tx(recv_bar, (uint32_t)((ns - 1) * my_own * kClChunkBytes));
        for (int d = 0; d < ns; ++d)
          if (d != sp) mbar_arrive_cluster(mapa_shared(smem_u32(free_bar), (uint32_t)d));
        ok = mbar_wait_cluster(free_bar, 0, err);
        B200_TL(10);
      }
      if (ok) {
        int off = 0;
        for (int d = 0; d < ns; ++d) {
          const int nd = n_own_of(d);
          if (d == sp || nd == 0) continue;  // (more splits than chunks: d owns none)
          const int src_slot = sp < d ? sp : sp - 1;
          const uint32_t dst = mapa_shared(
              smem_u32(smem + (size_t)recv_chunk(d, src_slot, 0) * kClChunkBytes), (uint32_t)d);
          bulk_copy_to_cluster(dst, smem + (size_t)off * kClChunkBytes,
                               (uint32_t)(nd * kClChunkBytes),
                               mapa_shared(smem_u32(recv_bar), (uint32_t)d));
          off += nd;
        }
      }
      *last_flag = ok ? 1 : 0;
    }
    named_barrier_sync(1, 128);
    const bool ok = *last_flag != 0 && mbar_wait(recv_bar, 0, err);
    if (etid == 0) B200_TL(13);
    if (!ok) {
      *abort_flag = 1;
    } else {
      tc_fence_after();
      int ebuf = 0;
#pragma unroll 1
      for (int k = 0; k < my_own; ++k) {
        const int ch = sp + k * ns;
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_acc + ch * 32, r);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) v[c] = 0.f;
        for (int s2 = 0; s2 < ns; ++s2) {
          if (s2 == sp) {
#pragma unroll
            for (int c = 0; c < 32; ++c) v[c] += __uint_as_float(r[c]);
          } else {
            const float4* src =
                reinterpret_cast<const float4*>(
                    smem + (size_t)recv_chunk(sp, s2 < sp ? s2 : s2 - 1, k) * kClChunkBytes) +
                row_in_tile * 8;
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) {
              const float4 x = src[c4 ^ (row_in_tile & 7)];
              v[4 * c4] += x.x;
              v[4 * c4 + 1] += x.y;
              v[4 * c4 + 2] += x.z;
              v[4 * c4 + 3] += x.w;
            }
          }
        }
        // bf16 tile store through the output map (64-byte rows, 64B swizzle).
        uint8_t* buf = epi_stage + (size_t)(q * 2 + ebuf) * 2048;
        if (lane == 0) bulk_wait_read_le1();
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 pk;
          pk.x = pack_bf16x2(v[8 * u + 0], v[8 * u + 1]);
          pk.y = pack_bf16x2(v[8 * u + 2], v[8 * u + 3]);
          pk.z = pack_bf16x2(v[8 * u + 4], v[8 * u + 5]);
          pk.w = pack_bf16x2(v[8 * u + 6], v[8 * u + 7]);
          *reinterpret_cast<uint4*>(buf + lane * 64 + ((u ^ ((lane >> 1) & 3)) * 16)) = pk;
        }
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmap_c, buf, uc.out_j0 + ch * 32, uc.out_i0 + q * 32);
          bulk_commit();
        }
        ebuf ^= 1;
      }
      if (lane == 0) bulk_wait_all();
    }
  }
  }
  if constexpr (CL) {
  if (!cl_bulk) {
    // -------------------------------------------------- cluster reduction
    // Rows of the tile are dealt out to the cluster's CTAs (CTA d owns rows
    // [d * R, (d + 1) * R)). Barrier 1: every CTA's MMAs are complete, so the
    // operand rings (reused as receive buffers) are idle. Each epilogue thread
    // then pushes its accumulator row straight from TMEM into the owner's
    // receive slot [split][row] with remote shared-memory stores (posted: no
    // round trip is exposed). Barrier 2: all rows have landed; each CTA sums
    // its rows over the splits in split order (the workspace path's fixed
    // order), applies the epilogue and stores bf16. No CTA touches another's
    // shared memory after barrier 2, so exiting is safe.
    constexpr int CW = BN % 32 == 0 ? 32 : 16;
    constexpr int LDP = BN + 4;  // padded row (floats): conflict-free 16-byte accesses
    static_assert((BMT + kMaxSplits) * LDP * 4 <= S::kTileBytes, "receive buffer exceeds the ring");
    static_assert(EPI != kEpiSiluMul || BN % 128 == 0, "SiLU tiles hold whole gate/up blocks");
    cluster_sync_all();
    if (cl_ok && warp >= 2) {
      const int q = warp & 3;
      const int row_in_tile = q * 32 + lane;
      const int nsplit = splits;
      const int R = (BMT + nsplit - 1) / nsplit;
      const uint32_t rank = cluster_ctarank();
      const uint32_t recv = smem_u32(smem);
#pragma unroll 1
      for (int h = 0; h < MH; ++h) {
        const int row = h * BM + row_in_tile;
        const int dst_cta = row / R;
        const uint32_t slot = (uint32_t)(((int)rank * R + (row - dst_cta * R)) * LDP);
        const uint32_t dst = mapa_shared(recv + slot * 4u, (uint32_t)dst_cta);
        const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + h * kHalfCols;
#pragma unroll 1
        for (int ch = 0; ch < BN / CW; ++ch) {
          uint32_t r[32];
          if constexpr (CW == 32) {
            tmem_ld_32x32b_x32(t_row + ch * CW, r);
          } else {
            tmem_ld_32x32b_x16(t_row + ch * CW, *reinterpret_cast<uint32_t(*)[16]>(r));
          }
          tmem_wait_ld();
#pragma unroll
          for (int v = 0; v < CW / 4; ++v)
            st_dsmem_f4(dst + (uint32_t)((ch * CW + 4 * v) * 4),
                        make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                    __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3])));
        }
      }
    }
    cluster_sync_all();
    if (!*abort_flag && (int)blockIdx.x < num_units) {
      constexpr int LDP = BN + 4;
      const int nsplit = splits;
      const int rank = (int)cluster_ctarank();
      const int t = (int)blockIdx.x / nsplit;
      const UnitCoord uc = unit_coord<BN>(t, num_m, num_n, grp, p_rows, q_rows, p_tile);
      const int R = (BMT + nsplit - 1) / nsplit;
      const int r0 = rank * R, r1 = min(BMT, r0 + R);
      // Receive slots: split s's copy of owned row r sits at (s * R + r - r0).
      const float* recv = reinterpret_cast<const float*>(smem);
      if constexpr (EPI == kEpiSiluMul) {
        // Columns hold [gate 64 | up 64] blocks: 16 output float4 groups per block.
        constexpr int G4 = BN / 8;
        const int out_j0 = (uc.q_row / BN) * (BN / 2);
        const int out_cols = q_rows / 2;
        for (int idx = threadIdx.x; idx < (r1 - r0) * G4; idx += blockDim.x) {
          const int r = r0 + idx / G4;
          const int o4 = idx % G4;
          const int gcol = (o4 / 16) * 128 + (o4 % 16) * 4;
          float4 g = make_float4(0.f, 0.f, 0.f, 0.f), uu = g;
#pragma unroll
          for (int sidx = 0; sidx < kMaxSplits; ++sidx) {
            if (sidx < nsplit) {
              const float* rowp = recv + (size_t)(sidx * R + r - r0) * LDP;
              const float4 a = *reinterpret_cast<const float4*>(rowp + gcol);
              const float4 b = *reinterpret_cast<const float4*>(rowp + gcol + 64);
              g.x += a.x; g.y += a.y; g.z += a.z; g.w += a.w;
              uu.x += b.x; uu.y += b.y; uu.z += b.z; uu.w += b.w;
            }
          }
          const int i = uc.out_i0 + r;
          const int j = out_j0 + (o4 / 16) * 64 + (o4 % 16) * 4;
          if ((MH == 2 || r < p_rows_tile) && i < p_rows && j < out_cols) {
            uint2 pk;
            pk.x = pack_bf16x2(__fdividef(g.x, 1.0f + __expf(-g.x)) * uu.x,
                               __fdividef(g.y, 1.0f + __expf(-g.y)) * uu.y);
            pk.y = pack_bf16x2(__fdividef(g.z, 1.0f + __expf(-g.z)) * uu.z,
                               __fdividef(g.w, 1.0f + __expf(-g.w)) * uu.w);
            *reinterpret_cast<uint2*>(C + (size_t)i * ldc + j) = pk;
          }
        }
      } else {
        constexpr int G4 = BN / 4;
        for (int idx = threadIdx.x; idx < (r1 - r0) * G4; idx += blockDim.x) {
          const int r = r0 + idx / G4;
          const int c4 = idx % G4;
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int sidx = 0; sidx < kMaxSplits; ++sidx) {
            if (sidx < nsplit) {
              const float4 a = *reinterpret_cast<const float4*>(
                  recv + (size_t)(sidx * R + r - r0) * LDP + c4 * 4);
              acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
            }
          }
          const int i = uc.out_i0 + r;
          const int j = uc.out_j0 + c4 * 4;
          if ((MH == 2 || r < p_rows_tile) && i < p_rows && j < q_rows) {
            uint2 pk;
            pk.x = pack_bf16x2(acc.x, acc.y);
            pk.y = pack_bf16x2(acc.z, acc.w);
            *reinterpret_cast<uint2*>(C + (size_t)i * ldc + j) = pk;
          }
        }
      }
    }
  }
  }

  if (threadIdx.x == 64) B200_TL(6);
  tc_fence_before();
  __syncthreads();
  // Pair / cluster split: no CTA may leave while a peer can still signal its
  // barriers or copy into or out of its shared memory; the TMEM release is
  // collective over a pair.
  if constexpr (PAIR || CL) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, kTmemCols);
    else tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0) B200_TL(7);
  if (ag_on && threadIdx.x == 0) {
    // Every CTA is past its waits: the last one hands the next launch its epoch.
    const uint32_t n = atomicAdd(wq.ag.pad_local + kAgPadDone, 1u) + 1u;
    if (n == gridDim.x) {
      atomicExch(wq.ag.pad_local + kAgPadDone, 0u);
      atomicExch(wq.ag.pad_local + kAgPadEpoch, ag_e);
    }
  }
  if constexpr (EPI == kEpiArNorm) {
    // Fused TP collective: every tile of this rank's stage is stored once all
    // CTAs have arrived; the same CTAs then all-reduce, add the residual and
    // RMS-normalise the rows this rank owns (peer loads / stores over NVLink).
    __shared__ float ar_part[ardev::kMaxVec * kThreads];
    __shared__ float ar_bcast;
    __shared__ int ar_ok;
    if (!*abort_flag) ardev::run_any(wq.ar, /*gated=*/true, ar_part, &ar_bcast, &ar_ok);
  }
#undef B200_TL
}

// Process-wide split-K workspace per device (fp32 partial tiles + arrival
// counters that the last-arriving CTA re-arms). Configured once at start-up.
struct SplitWorkspace {
  float* ws = nullptr;
  size_t ws_bytes = 0;
  int* counters = nullptr;
  int n_counters = 0;
};
SplitWorkspace g_split_ws[64];

// Rows per TMA box for the bf16 operands (VLLM_B200_GEMM_TMA_BOX; 0 = whole tile).
int tma_box_rows() {
  static const int v = [] {
    const char* e = std::getenv("VLLM_B200_GEMM_TMA_BOX");
    return e ? std::atoi(e) : 0;
  }();
  return v;
}

// Split-K reduction mode: VLLM_B200_GEMM_SERIAL_SPLIT=1 makes the last split
// to arrive sum each tile (the others exit early); default: the splits of a
// tile that are resident together share the reduction.
bool serial_split_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("VLLM_B200_GEMM_SERIAL_SPLIT");
    return e != nullptr && e[0] == '1';
  }();
  return on;
}
int split_arg(int splits) {
  return (splits > 1 && serial_split_enabled()) ? (splits | kSerialSplitFlag) : splits;
}

template <int BN, int STAGES, bool SWAP, int EPI, int WF = kWBf16, int MH = 1>
bool launch_cfg(const void* P, const void* Q, void* C, int p_rows, int q_rows, int K, int ldp,
                int ldq, int ldc, int splits, float* ws, int* counters, unsigned int* err,
                cudaStream_t stream, const WQParams& wq = WQParams{},
                const GroupInfo& grp = GroupInfo{}, int grid_units = 0, int pm = BM,
                bool ext = false, int p_map_rows = 0) {
  using S = Smem<BN, STAGES, WF, MH>;
  if (MH != 1 || WF != kWBf16 || grp.E > 0 || pm <= 0 || pm > BM) pm = BM;
  // TMA box rows per operand (bf16 operands only; 0 = one box per tile).
  int pbox = pm, qbox = BN;
  if (WF == kWBf16) {
    const int want = tma_box_rows();
    if (want > 0 && pm % want == 0) pbox = want;
    if (want > 0 && BN % want == 0) qbox = want;
  }
  static_assert(S::kTotal <= 232448, "shared memory budget");
  auto kernel = gemm_bf16_tc_kernel<BN, STAGES, SWAP, EPI, WF, MH>;
  static bool attr_set[kMaxDevices] = {};  // per instantiation and device; idempotent if raced
  set_smem_attr_once(kernel, S::kTotal, attr_set, "gemm_bf16_tc");
  CUtensorMap tp;
  if constexpr (WF == kWBf16) {
    // (p_map_rows: the map spans more rows than are tiled -- the two halves
    // of an all-gather buffer)
    tp = make_tmap_2d(P, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p_map_rows > 0 ? p_map_rows : p_rows,
                      K, (uint64_t)ldp * 2, pbox, BK);
  } else {
    // Raw quantised rows: K * bytes-per-element bytes, box = 128 rows x one k-block.
    const int rb = raw_row_bytes(WF);
    tp = make_tmap_2d(P, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p_rows, (uint64_t)K * rb / 64,
                      (uint64_t)ldp, BM, rb, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  CUtensorMap tq = make_tmap_2d(Q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q_rows, K,
                                (uint64_t)ldq * 2, qbox, BK);
  // Output map for the epilogue's tile stores (plain normal-mode bf16 only;
  // other instantiations never read it and get the operand map instead).
  constexpr int kCW = BN % 32 == 0 ? 32 : 16;
  const CUtensorMap tc_plain =
      (EPI == kEpiNone && !SWAP && WF == kWBf16)
          ? make_tmap_2d(C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p_rows, q_rows, (uint64_t)ldc * 2,
                         32, kCW, kCW == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B)
          : tq;
  const CUtensorMap tc =
      ext ? make_tmap_3d(ws, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)splits, p_rows, q_rows,
                         (uint64_t)q_rows * 4, (uint64_t)p_rows * q_rows * 4, 1, 32, 32)
          : tc_plain;
  int dev = 0;
  cudaGetDevice(&dev);
  const int p_stride = MH == 1 ? pm : BM * MH;
  const long units = grid_units > 0 ? grid_units
                                    : (long)((p_rows + p_stride - 1) / p_stride) *
                                          ((q_rows + BN - 1) / BN) * splits;
  const int grid = units < num_sms(dev) ? (int)units : num_sms(dev);
  // One round (every unit resident at once) and the kernel's staging fits.
  constexpr bool kExtFits = EPI == kEpiNone && !SWAP && WF == kWBf16 && BN % 32 == 0 &&
                            MH * BN * BM * 4 <= S::kTileBytes;
  const bool use_ext = kExtFits && ext && splits > 1 && units <= grid;
  WQParams q = wq;
  if (WF == kWBf16) q.out_scale = 1.f;
  launch_pdl(kernel, dim3(grid), dim3(WF == kWBf16 ? kThreads : kThreadsQ), S::kTotal, stream,
             nullptr, tp, tq, use_ext ? tc : tc_plain, reinterpret_cast<__nv_bfloat16*>(C), ldc, p_rows,
             q_rows, K, use_ext ? -splits : split_arg(splits), ws, counters, err, q, grp, pm,
             pbox, qbox);
  return use_ext;
}

// Cluster split-K: the `splits` K-slices of a tile run as one thread-block
// cluster (one tile-split per CTA, grid = tiles * splits) and reduce through
// distributed shared memory; no workspace or counters.
template <int BN, int STAGES, int EPI, int MH>
bool launch_cl(const void* A, const void* W, void* C, int M, int N, int K, int lda, int ldw,
               int ldc, int splits, unsigned int* err, cudaStream_t stream) {
  using S = Smem<BN, STAGES, kWBf16, MH>;
  static_assert(S::kTotal <= 232448, "shared memory budget");
  auto kernel = gemm_bf16_tc_kernel<BN, STAGES, false, EPI, kWBf16, MH, true>;
  static bool attr_set[kMaxDevices] = {};  // per instantiation and device; idempotent if raced
  set_smem_attr_once(kernel, S::kTotal, attr_set, "gemm_bf16_tc");
  CUtensorMap tp = make_tmap_2d(A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, (uint64_t)lda * 2,
                                BM, BK);
  CUtensorMap tq = make_tmap_2d(W, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, (uint64_t)ldw * 2,
                                BN, BK);
  // Output map for the bulk-copy reduction's tile stores (32 rows x 32 bf16,
  // 64-byte swizzle); other instantiations never read it.
  const CUtensorMap tc =
      (EPI == kEpiNone && MH == 1 && BN % 32 == 0)
          ? make_tmap_2d(C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, N, (uint64_t)ldc * 2, 32, 32,
                         CU_TENSOR_MAP_SWIZZLE_64B)
          : tq;
  const long tiles = (long)((M + BM * MH - 1) / (BM * MH)) * ((N + BN - 1) / BN);
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3((unsigned)(tiles * splits), 1, 1);
  lc.blockDim = dim3(kThreads, 1, 1);
  lc.dynamicSmemBytes = S::kTotal;
  lc.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = pdl_enabled() ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&lc, kernel, tp, tq, tc, reinterpret_cast<__nv_bfloat16*>(C),
                                     ldc, M, N, K, splits, (float*)nullptr, (int*)nullptr, err,
                                     WQParams{}, GroupInfo{}, (int)BM, (int)BM, BN);
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("gemm_bf16_tc cluster launch: ") + cudaGetErrorString(e));
  return false;
}

// CTA pairs: cluster of 2, grid = 2 x min(units, SMs / 2), each pair
// persistent over (256 x BN tile, split) units; split-K through the workspace
// with one arrival counter per tile half (needs 2 x tiles counters).
template <int BN, int STAGES, int EPI>
bool launch_pair(const void* A, const void* W, void* C, int M, int N, int K, int lda, int ldw,
                 int ldc, int splits, float* ws, int* counters, unsigned int* err,
                 cudaStream_t stream, bool ext = false) {
  using S = Smem<BN / 2, STAGES, kWBf16, 1>;
  static_assert(S::kTotal <= 232448, "shared memory budget");
  auto kernel = gemm_bf16_tc_kernel<BN, STAGES, false, EPI, kWBf16, 1, false, true>;
  static bool attr_set[kMaxDevices] = {};  // per instantiation and device; idempotent if raced
  set_smem_attr_once(kernel, S::kTotal, attr_set, "gemm_bf16_tc");
  CUtensorMap tp = make_tmap_2d(A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, (uint64_t)lda * 2,
                                BM, BK);
  CUtensorMap tq = make_tmap_2d(W, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, (uint64_t)ldw * 2,
                                BN / 2, BK);
  constexpr int kCW = BN % 32 == 0 ? 32 : 16;
  const CUtensorMap tc_plain =
      EPI == kEpiNone
          ? make_tmap_2d(C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, N, (uint64_t)ldc * 2, 32, kCW,
                         kCW == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B)
          : tq;
  const CUtensorMap tc =
      ext ? make_tmap_3d(ws, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)splits, M, N,
                         (uint64_t)N * 4, (uint64_t)M * N * 4, 1, 32, 32)
          : tc_plain;
  int dev = 0;
  cudaGetDevice(&dev);
  const long units = (long)((M + 2 * BM - 1) / (2 * BM)) * ((N + BN - 1) / BN) * splits;
  cudaLaunchConfig_t lc = {};
  lc.blockDim = dim3(kThreads, 1, 1);
  lc.dynamicSmemBytes = S::kTotal;
  lc.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;  // occupancy query: cluster shape only
  // Pairs that can be resident at once (the GPC layout can leave SMs
  // unpairable); the persistent grid never exceeds it, so every pair runs
  // concurrently (the co-resident split-K reduction relies on it).
  static int max_pairs[64] = {0};
  if (max_pairs[dev] == 0) {
    lc.gridDim = dim3((unsigned)(2 * (num_sms(dev) / 2)), 1, 1);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (void*)kernel, &lc) != cudaSuccess || n <= 0)
      n = num_sms(dev) / 2;
    cudaGetLastError();
    max_pairs[dev] = n < num_sms(dev) / 2 ? n : num_sms(dev) / 2;
  }
  const long pairs = units < max_pairs[dev] ? units : max_pairs[dev];
  // One round (every unit resident at once) and the kernel's staging fits.
  constexpr bool kExtFits = EPI == kEpiNone && BN % 32 == 0 && BN * BM * 4 <= S::kTileBytes;
  const bool use_ext = kExtFits && ext && splits > 1 && units <= pairs;
  lc.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  lc.numAttrs = pdl_enabled() ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&lc, kernel, tp, tq, use_ext ? tc : tc_plain,
                                     reinterpret_cast<__nv_bfloat16*>(C), ldc, M, N, K,
                                     use_ext ? -splits : split_arg(splits), ws, counters, err,
                                     WQParams{}, GroupInfo{},
                                     (int)BM, (int)BM, BN / 2);
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("gemm_bf16_tc pair launch: ") + cudaGetErrorString(e));
  return use_ext;
}

struct CfgInfo {
  int bn;
  bool swap;
  int mh;     // 128-row M halves per tile (2 = 256-row tall tile)
  bool cl;    // split-K as a cluster with a distributed-shared-memory reduction
  bool pair;  // CTA pair (cta_group::2): 256 x bn tile over two SMs
};
constexpr CfgInfo kCfgInfo[kCfgCount] = {
    {256, false, 1, false, false}, {128, false, 1, false, false}, {16, true, 1, false, false},
    {32, true, 1, false, false},   {64, true, 1, false, false},   {192, false, 1, false, false},
    {96, false, 1, false, false},  {64, false, 1, false, false},  {128, true, 1, false, false},
    {256, false, 2, false, false}, {224, false, 2, false, false}, {128, false, 2, false, false},
    {112, false, 2, false, false}, {64, false, 2, false, false},  {256, false, 1, true, false},
    {128, false, 1, true, false},  {128, false, 2, true, false},  {112, false, 2, true, false},
    {64, false, 2, true, false},   {256, false, 1, false, true},  {128, false, 1, false, true},
    {192, false, 1, false, true},  {64, false, 1, false, true},   {96, false, 1, false, true},
};

int cfg_bn(int cfg) { return (cfg >= 0 && cfg < kCfgCount) ? kCfgInfo[cfg].bn : 0; }

// Weight rows per swap-AB tile: the multiple of 8 in [32, 128] that minimises
// waves x (rows + token tile) -- fewer rows per tile spread the weights over
// more SMs when 128-row tiles would leave SMs idle or spill into a partial
// wave (e.g. 4096 rows x 4 token tiles: 112 rows -> 148 tiles, one full wave).
int swap_tile_rows(long p_rows, long q_tiles, int splits, int num_sm, int bn) {
  int best = 128;
  double best_cost = 1e30;
  for (int pm = 128; pm >= 32; pm -= 8) {
    const long units = ((p_rows + pm - 1) / pm) * q_tiles * splits;
    const long waves = (units + num_sm - 1) / num_sm;
    const double cost = (double)waves * (pm + bn);
    if (cost < best_cost * 0.999) {
      best_cost = cost;
      best = pm;
    }
  }
  return best;
}
bool cfg_swap(int cfg) { return cfg >= 0 && cfg < kCfgCount && kCfgInfo[cfg].swap; }
int cfg_mh(int cfg) { return (cfg >= 0 && cfg < kCfgCount) ? kCfgInfo[cfg].mh : 1; }
bool cfg_cl(int cfg) { return cfg >= 0 && cfg < kCfgCount && kCfgInfo[cfg].cl; }
bool cfg_pair(int cfg) { return cfg >= 0 && cfg < kCfgCount && kCfgInfo[cfg].pair; }
bool cfg_silu_ok(int cfg) {
  return cfg == kCfgN256 || cfg == kCfgN128 || cfg == kCfgM2N256 || cfg == kCfgM2N128 ||
         cfg == kCfgClN256 || cfg == kCfgClM2N128 || cfg == kCfgP2N256 || cfg == kCfgP2N128;
}

// Tuned dispatch table: (M, N, K, epi) -> plan, filled by the warm-up tuner
// or imported from a LUT file; consulted before the cost model.
struct PlanKey {
  int M, N, K, epi;
  bool operator==(const PlanKey& o) const {
    return M == o.M && N == o.N && K == o.K && epi == o.epi;
  }
};
struct PlanKeyHash {
  size_t operator()(const PlanKey& k) const {
    return ((size_t)k.M * 1000003u) ^ ((size_t)k.N * 10007u) ^ ((size_t)k.K * 131u) ^ k.epi;
  }
};
std::mutex g_plan_mu;
std::unordered_map<PlanKey, GemmPlan, PlanKeyHash> g_plans;

}  // namespace

int gemm_cfg_tile_n(int cfg) { return cfg_bn(cfg); }

void gemm_set_timeline(unsigned long long* buf) {
  cudaError_t e = cudaMemcpyToSymbol(g_gemm_timeline, &buf, sizeof(buf));
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("gemm_set_timeline: ") + cudaGetErrorString(e));
}
int gemm_cfg_tile_m(int cfg) { return cfg_pair(cfg) ? 256 : 128 * cfg_mh(cfg); }

SplitGeometry gemm_split_geometry(int M, int N, int K, int cfg, int splits, int num_sm) {
  SplitGeometry g;
  const int bn = cfg_bn(cfg);
  const bool swap = cfg_swap(cfg);
  const long p = swap ? N : M, qq = swap ? M : N;
  const long q_tiles = bn > 0 ? (qq + bn - 1) / bn : 0;
  g.tile_rows = gemm_cfg_tile_m(cfg);
  if (swap && bn > 0) g.tile_rows = swap_tile_rows(p, q_tiles, splits, num_sm, bn);
  g.tiles = ((p + g.tile_rows - 1) / g.tile_rows) * q_tiles;
  // fp32 partials are stored for whole 128-row (or 256-row) MMA tiles; a CTA
  // pair counts arrivals per tile half.
  g.ws_bytes = (size_t)g.tiles * splits * gemm_cfg_tile_m(cfg) * bn * sizeof(float);
  g.counters = cfg_pair(cfg) ? 2 * g.tiles : g.tiles;
  (void)K;
  return g;
}
bool gemm_cfg_is_cluster(int cfg) { return cfg_cl(cfg); }
bool gemm_cfg_is_swap(int cfg) { return cfg_swap(cfg); }

GemmPlan gemm_bf16_plan(int M, int N, int K, int epi, int num_sm) {
  {
    std::lock_guard<std::mutex> g(g_plan_mu);
    auto it = g_plans.find(PlanKey{M, N, K, epi});
    if (it != g_plans.end()) return it->second;
  }
  // Candidate tile shapes: swap-AB (weights on the 128-row side) for small M.
  int cands[24];
  int nc = 0;
  if (epi == kEpiNone && M <= 64) {
    cands[nc++] = M <= 16 ? kCfgSwap16 : (M <= 32 ? kCfgSwap32 : kCfgSwap64);
  } else if (epi == kEpiSiluMul) {
    cands[nc++] = kCfgN256;
    cands[nc++] = kCfgN128;
    if (M > 128) {
      cands[nc++] = kCfgM2N256;
      cands[nc++] = kCfgM2N128;
    }
    if (M > 128) {
      cands[nc++] = kCfgP2N256;
      cands[nc++] = kCfgP2N128;
    }
  } else {
    cands[nc++] = kCfgN256;
    cands[nc++] = kCfgN192;
    cands[nc++] = kCfgN128;
    cands[nc++] = kCfgN96;
    if (M > 128) {
      cands[nc++] = kCfgM2N256;
      cands[nc++] = kCfgM2N224;
      cands[nc++] = kCfgM2N128;
      cands[nc++] = kCfgM2N112;
    }
    if (M <= 256) {
      cands[nc++] = kCfgSwap64;
      cands[nc++] = kCfgSwap128;
    }
    if (M > 128) {
      cands[nc++] = kCfgP2N256;
      cands[nc++] = kCfgP2N192;
      cands[nc++] = kCfgP2N128;
      cands[nc++] = kCfgP2N96;
    }
  }
  const int num_kb = (K + 63) / 64;
  GemmPlan best{cands[0], 1};
  double best_cost = 1e30;
  for (int ci = 0; ci < nc; ++ci) {
    const int cfg = cands[ci];
    const int bn = cfg_bn(cfg);
    const int mh = cfg_mh(cfg);
    const bool cl = cfg_cl(cfg);
    for (int s = cl ? 2 : 1; s <= kMaxSplits; ++s) {
      const int kb_per = (num_kb + s - 1) / s;
      if (s > 1 && kb_per < 4) break;
      const SplitGeometry geo = gemm_split_geometry(M, N, K, cfg, s, num_sm);
      const long units = geo.tiles * s;
      const bool pair = cfg_pair(cfg);
      const int slots = pair ? num_sm / 2 : num_sm;  // a pair unit occupies two SMs
      const long waves = (units + slots - 1) / slots;
      // Relative cost model: a k-block costs the larger of its MMA time
      // (grows with the tile area) and its operand load time (grows with the
      // rows loaded), plus a fixed latency share, per-unit prologue /
      // epilogue, and the split partial-sum round trips.
      const double mma = mh * bn / 256.0;  // per SM
      const double load = pair ? (128.0 + bn / 2.0) / 384.0 * 0.8
                               : ((double)geo.tile_rows + bn) / 384.0 * 0.8;
      const double per_kb = (mma > load ? mma : load) + 0.25;
      double t_unit = kb_per * per_kb + 3.0 * mh;
      if (cl) t_unit += 1.5 + (mh * bn / 256.0);  // parallel reduction over the cluster
      else if (s > 1) t_unit += 4.0 + ((s + 3) / 4) * (mh * bn / 256.0) * 2.0;
      const double cost = waves * t_unit;
      if (cost < best_cost * 0.97) {
        best_cost = cost;
        best = {cfg, s};
      }
    }
  }
  return best;
}

void gemm_set_plan(int M, int N, int K, int epi, int cfg, int splits) {
  std::lock_guard<std::mutex> g(g_plan_mu);
  if (cfg < 0) {
    g_plans.erase(PlanKey{M, N, K, epi});
    return;
  }
  g_plans[PlanKey{M, N, K, epi}] = GemmPlan{cfg, splits < 1 ? 1 : splits};
}

void gemm_clear_plans() {
  std::lock_guard<std::mutex> g(g_plan_mu);
  g_plans.clear();
}

std::vector<int> gemm_export_plans() {
  std::lock_guard<std::mutex> g(g_plan_mu);
  std::vector<int> out;
  for (auto& kv : g_plans) {
    out.insert(out.end(), {kv.first.M, kv.first.N, kv.first.K, kv.first.epi, kv.second.cfg,
                           kv.second.splits});
  }
  return out;
}

int gemm_bf16_pick_config(int M, int N, int K, int epi, int num_sm) {
  return gemm_bf16_plan(M, N, K, epi, num_sm).cfg;
}

void gemm_configure_workspace(int device, size_t ws_bytes, int n_counters) {
  SplitWorkspace& w = g_split_ws[device];
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  if (w.ws) cudaFree(w.ws);
  if (w.counters) cudaFree(w.counters);
  w = SplitWorkspace{};
  cudaError_t e = cudaSuccess;
  if (ws_bytes > 0) e = cudaMalloc(&w.ws, ws_bytes);
  if (e == cudaSuccess && n_counters > 0) e = cudaMalloc(&w.counters, sizeof(int) * n_counters);
  if (e == cudaSuccess && n_counters > 0) e = cudaMemset(w.counters, 0, sizeof(int) * n_counters);
  cudaSetDevice(prev);
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("gemm workspace: ") + cudaGetErrorString(e));
  w.ws_bytes = ws_bytes;
  w.n_counters = n_counters;
}

size_t gemm_workspace_bytes(int device) { return g_split_ws[device].ws_bytes; }
float* gemm_ws_ptr(int device) { return g_split_ws[device].ws; }
int* gemm_counters_ptr(int device) { return g_split_ws[device].counters; }
int gemm_n_counters(int device) { return g_split_ws[device].n_counters; }

namespace {

// Returns true when the launched GEMM left its split-K partials in the
// workspace for splitk_reduce_kernel (external reduction, `ext_req`).
bool launch_split_impl(const void* A, const void* W, void* C, int M, int N, int K, int lda,
                       int ldw, int ldc, int epi, int cfg, int splits, float* ws, size_t ws_bytes,
                       int* counters, int n_counters, unsigned int* err, cudaStream_t stream,
                       bool ext_req) {
  if (M <= 0 || N <= 0 || K <= 0) return false;
  if (K % 8 != 0 || lda % 8 != 0 || ldw % 8 != 0)
    throw std::runtime_error("gemm_bf16: K and leading dims must be multiples of 8");
  if (N % 8 != 0 || ldc % 8 != 0) throw std::runtime_error("gemm_bf16: N, ldc must be multiples of 8");
  int dev = 0;
  cudaGetDevice(&dev);
  if (cfg < 0) {
    GemmPlan pl = gemm_bf16_plan(M, N, K, epi, num_sms(dev));
    cfg = pl.cfg;
    if (splits <= 0) splits = pl.splits;
  }
  if (splits <= 0) splits = 1;
  if (splits > kMaxSplits) splits = kMaxSplits;
  if (epi == kEpiSiluMul && !cfg_silu_ok(cfg)) cfg = kCfgN128;
  const int bn = cfg_bn(cfg);
  if (bn == 0) throw std::runtime_error("gemm_bf16: unknown config " + std::to_string(cfg));
  const int num_kb = (K + 63) / 64;
  if (splits > num_kb) splits = num_kb;
  if (cfg_cl(cfg)) {
    if (epi == kEpiSiluMul && N % 128 != 0)
      throw std::runtime_error("gemm_bf16 silu_mul: N must be a multiple of 128");
    if (splits > 1) {
      if (epi == kEpiSiluMul) {
        if (cfg == kCfgClN256)
          return launch_cl<256, 4, kEpiSiluMul, 1>(A, W, C, M, N, K, lda, ldw, ldc, splits, err,
                                                   stream);
        return launch_cl<128, 4, kEpiSiluMul, 2>(A, W, C, M, N, K, lda, ldw, ldc, splits, err,
                                                 stream);
      }
      switch (cfg) {
        case kCfgClN256:
          return launch_cl<256, 4, kEpiNone, 1>(A, W, C, M, N, K, lda, ldw, ldc, splits, err, stream);
        case kCfgClN128:
          return launch_cl<128, 6, kEpiNone, 1>(A, W, C, M, N, K, lda, ldw, ldc, splits, err, stream);
        case kCfgClM2N128:
          return launch_cl<128, 4, kEpiNone, 2>(A, W, C, M, N, K, lda, ldw, ldc, splits, err, stream);
        case kCfgClM2N112:
          return launch_cl<112, 4, kEpiNone, 2>(A, W, C, M, N, K, lda, ldw, ldc, splits, err, stream);
        case kCfgClM2N64:
          return launch_cl<64, 5, kEpiNone, 2>(A, W, C, M, N, K, lda, ldw, ldc, splits, err, stream);
      }
    }
    // One K slice: the plain persistent tile of the same shape.
    cfg = cfg == kCfgClN256 ? kCfgN256 : cfg == kCfgClN128 ? kCfgN128
        : cfg == kCfgClM2N128 ? kCfgM2N128 : cfg == kCfgClM2N112 ? kCfgM2N112 : kCfgM2N64;
    splits = 1;
  }
  SplitGeometry geo = gemm_split_geometry(M, N, K, cfg, splits, num_sms(dev));
  if (splits > 1 && (ws == nullptr || geo.ws_bytes > ws_bytes || geo.counters > n_counters)) {
    splits = 1;  // no room: no split
    geo = gemm_split_geometry(M, N, K, cfg, splits, num_sms(dev));
  }
  const int pm = geo.tile_rows;
  float* wsp = splits > 1 ? ws : nullptr;
  int* cnt = splits > 1 ? counters : nullptr;
  const bool ext = ext_req && splits > 1 && epi == kEpiNone && ws != nullptr &&
                   (size_t)splits * M * N * sizeof(float) <= ws_bytes;
  if (cfg_pair(cfg) && epi == kEpiSiluMul) {
    if (N % 128 != 0) throw std::runtime_error("gemm_bf16 silu_mul: N must be a multiple of 128");
    if (cfg == kCfgP2N256)
      return launch_pair<256, 6, kEpiSiluMul>(A, W, C, M, N, K, lda, ldw, ldc, splits, wsp, cnt,
                                              err, stream);
    return launch_pair<128, 8, kEpiSiluMul>(A, W, C, M, N, K, lda, ldw, ldc, splits, wsp, cnt, err,
                                            stream);
  }
  if (cfg_pair(cfg)) {
    switch (cfg) {
      case kCfgP2N256:
        return launch_pair<256, 6, kEpiNone>(A, W, C, M, N, K, lda, ldw, ldc, splits, wsp, cnt, err,
                                             stream, ext);
      case kCfgP2N192:
        return launch_pair<192, 7, kEpiNone>(A, W, C, M, N, K, lda, ldw, ldc, splits, wsp, cnt, err,
                                             stream, ext);
      case kCfgP2N128:
        return launch_pair<128, 8, kEpiNone>(A, W, C, M, N, K, lda, ldw, ldc, splits, wsp, cnt, err,
                                             stream, ext);
      case kCfgP2N96:
        return launch_pair<96, 9, kEpiNone>(A, W, C, M, N, K, lda, ldw, ldc, splits, wsp, cnt, err,
                                            stream, ext);
      default:
        return launch_pair<64, 10, kEpiNone>(A, W, C, M, N, K, lda, ldw, ldc, splits, wsp, cnt, err,
                                             stream, ext);
    }
  }
  if (epi == kEpiSiluMul) {
    if (N % 128 != 0) throw std::runtime_error("gemm_bf16 silu_mul: N must be a multiple of 128");
    if (cfg == kCfgN256)
      return launch_cfg<256, 4, false, kEpiSiluMul>(A, W, C, M, N, K, lda, ldw, ldc, splits, wsp,
                                                    cnt, err, stream);
    if (cfg == kCfgM2N256)
      return launch_cfg<256, 3, false, kEpiSiluMul, kWBf16, 2>(A, W, C, M, N, K, lda, ldw, ldc,
                                                               splits, wsp, cnt, err, stream);
    if (cfg == kCfgM2N128)
      return launch_cfg<128, 4, false, kEpiSiluMul, kWBf16, 2>(A, W, C, M, N, K, lda, ldw, ldc,
                                                               splits, wsp, cnt, err, stream);
    return launch_cfg<128, 6, false, kEpiSiluMul>(A, W, C, M, N, K, lda, ldw, ldc, splits, wsp,
                                                  cnt, err, stream);
  }
#define B200_NORMAL(BN_, ST_) \
  return launch_cfg<BN_, ST_, false, kEpiNone>(A, W, C, M, N, K, lda, ldw, ldc, splits, wsp, cnt, \
                                               err, stream, WQParams{}, GroupInfo{}, 0, pm, ext)
#define B200_TALL(BN_, ST_) \
  return launch_cfg<BN_, ST_, false, kEpiNone, kWBf16, 2>(A, W, C, M, N, K, lda, ldw, ldc, splits, \
                                                          wsp, cnt, err, stream, WQParams{},     \
                                                          GroupInfo{}, 0, BM, ext)
#define B200_SWAP(BN_, ST_) \
  return launch_cfg<BN_, ST_, true, kEpiNone>(W, A, C, N, M, K, ldw, lda, ldc, splits, wsp, cnt, \
                                              err, stream, WQParams{}, GroupInfo{}, 0, pm)
  switch (cfg) {
    case kCfgN256: B200_NORMAL(256, 4);
    case kCfgN192: B200_NORMAL(192, 5);
    case kCfgN128: B200_NORMAL(128, 6);
    case kCfgN96: B200_NORMAL(96, 7);
    case kCfgN64: B200_NORMAL(64, 8);
    case kCfgSwap16: B200_SWAP(16, 8);
    case kCfgSwap32: B200_SWAP(32, 8);
    case kCfgSwap64: B200_SWAP(64, 8);
    case kCfgSwap128: B200_SWAP(128, 6);
    case kCfgM2N256: B200_TALL(256, 3);
    case kCfgM2N224: B200_TALL(224, 3);
    case kCfgM2N128: B200_TALL(128, 4);
    case kCfgM2N112: B200_TALL(112, 4);
    case kCfgM2N64: B200_TALL(64, 5);
  }
#undef B200_TALL
#undef B200_NORMAL
#undef B200_SWAP
  return false;
}

// Opt-in (VLLM_B200_GEMM_EXT_REDUCE=1): measured on the Llama-3.1-8B decode
// shapes it shortened the GEMM kernel's epilogue from about 8 to 3.6 us, but
// the reduction kernel that follows took the difference back (qkv M = 256:
// 29.6 vs 28.7 us per call; decode phase 3,227 vs 3,201 ms per bench step).
bool ext_reduce_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("VLLM_B200_GEMM_EXT_REDUCE");
    return e != nullptr && e[0] == '1';
  }();
  return on;
}

// C[m, n] = bf16(sum over s in order 0, 1, ... of ws[s][m][n]): the split
// partials the GEMM left in the workspace; 8 columns per thread.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int M, int N,
                                     __nv_bfloat16* __restrict__ C, int ldc) {
  pdl_wait();
  const long n8 = N / 8;
  const long total = (long)M * n8;
  for (long idx = (long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long)gridDim.x * blockDim.x) {
    const int m = (int)(idx / n8), c = (int)(idx - (long)m * n8) * 8;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int sp = 0; sp < splits; ++sp) {
      const float4* src = reinterpret_cast<const float4*>(ws + ((size_t)sp * M + m) * N + c);
      const float4 a = __ldcg(src), b = __ldcg(src + 1);
      v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
      v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
    }
    uint4 pk;
    pk.x = pack_bf16x2(v[0], v[1]);
    pk.y = pack_bf16x2(v[2], v[3]);
    pk.z = pack_bf16x2(v[4], v[5]);
    pk.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(C + (size_t)m * ldc + c) = pk;
  }
}

}  // namespace

void gemm_bf16_launch_split(const void* A, const void* W, void* C, int M, int N, int K, int lda,
                            int ldw, int ldc, int epi, int cfg, int splits, float* ws,
                            size_t ws_bytes, int* counters, int n_counters, unsigned int* err,
                            cudaStream_t stream, bool ext_reduce) {
  const bool ext_req = ext_reduce && ext_reduce_enabled();
  if (!launch_split_impl(A, W, C, M, N, K, lda, ldw, ldc, epi, cfg, splits, ws, ws_bytes,
                         counters, n_counters, err, stream, ext_req))
    return;
  // The GEMM wrote split partials [splits][M][N]; splits as the launcher resolved them.
  int dev = 0;
  cudaGetDevice(&dev);
  int s = splits;
  if (cfg < 0 || s <= 0) s = gemm_bf16_plan(M, N, K, epi, num_sms(dev)).splits;
  if (s > kMaxSplits) s = kMaxSplits;
  const int num_kb = (K + 63) / 64;
  if (s > num_kb) s = num_kb;
  const long total = (long)M * (N / 8);
  const long blocks = (total + 255) / 256;
  const int grid = (int)(blocks < 8L * num_sms(dev) ? blocks : 8L * num_sms(dev));
  launch_pdl(splitk_reduce_kernel, dim3(grid), dim3(256), 0, stream, nullptr, ws, s, M, N,
             reinterpret_cast<__nv_bfloat16*>(C), ldc);
}


// All-gather -> GEMM: C[T, N] = gather(shards)[T, K] . W^T with the gather
// inside the GEMM (AgParams). Tiles are plain normal-mode tiles (128 x 256 or
// 128 x 128, or the 256-row tall ones), split-K as planned.
void gemm_ag_launch(const void* W, void* C, int T, int N, int K, int ldw, int ldc, int cfg,
                    int splits, const AgParams& ag, unsigned int* err, cudaStream_t stream) {
  if (ag.world < 2 || ag.world > kMaxRanks || T != ag.rows_per_rank * ag.world || T > ag.t_max ||
      K != ag.K || K % 8 != 0)
    throw std::runtime_error("gemm_ag: bad shape / world");
  int dev = 0;
  cudaGetDevice(&dev);
  if (cfg < 0) {
    const GemmPlan pl = gemm_bf16_plan(T, N, K, kEpiNone, num_sms(dev));
    cfg = pl.cfg;
    if (splits <= 0) splits = pl.splits;
  }
  if (splits <= 0) splits = 1;
  // The gather needs plain normal-mode tiles.
  if (cfg == kCfgM2N224 || cfg == kCfgM2N112 || cfg == kCfgP2N256 || cfg == kCfgClM2N128 ||
      cfg == kCfgClM2N112)
    cfg = kCfgM2N128;
  else if (cfg == kCfgM2N64 || cfg == kCfgClM2N64)
    cfg = kCfgM2N128;
  else if (cfg != kCfgN256 && cfg != kCfgN128 && cfg != kCfgM2N256 && cfg != kCfgM2N128)
    cfg = kCfgN128;
  SplitWorkspace& ws = g_split_ws[dev];
  SplitGeometry geo = gemm_split_geometry(T, N, K, cfg, splits, num_sms(dev));
  if (splits > 1 && (ws.ws == nullptr || geo.ws_bytes > ws.ws_bytes || geo.counters > ws.n_counters))
    splits = 1;
  float* wsp = splits > 1 ? ws.ws : nullptr;
  int* cnt = splits > 1 ? ws.counters : nullptr;
  WQParams wq{};
  wq.ag = ag;
  const void* P = ag.xfull_peer[ag.rank];
  const int map_rows = 2 * ag.t_max;
#define B200_AG(BN_, ST_, MH_)                                                                   \
  launch_cfg<BN_, ST_, false, kEpiNone, kWBf16, MH_>(P, W, C, T, N, K, K, ldw, ldc, splits, wsp, \
                                                    cnt, err, stream, wq, GroupInfo{}, 0, BM,   \
                                                    false, map_rows);                           \
  return
  switch (cfg) {
    case kCfgN256: B200_AG(256, 4, 1);
    case kCfgM2N256: B200_AG(256, 3, 2);
    case kCfgM2N128: B200_AG(128, 4, 2);
    default: B200_AG(128, 6, 1);
  }
#undef B200_AG
}

bool gemm_ar_rmsnorm_launch(const void* A, const void* W, int M, int N, int K, int lda, int ldw,
                            int cfg, int splits, const ArRmsNormParams& ar, unsigned int* err,
                            cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return true;
  if (M != ar.T || N != ar.H || K % 8 != 0 || lda % 8 != 0 || ldw % 8 != 0 || N % 8 != 0)
    return false;
  if ((ar.world != 1 && ar.world != 2 && ar.world != 4 && ar.world != 8) ||
      N / 8 > ardev::kMaxVec * kThreads)
    return false;
  int dev = 0;
  cudaGetDevice(&dev);
  if (cfg < 0) {
    GemmPlan pl = gemm_bf16_plan(M, N, K, kEpiNone, num_sms(dev));
    cfg = pl.cfg;
    if (splits <= 0) splits = pl.splits;
  }
  if (splits <= 0) splits = 1;
  if (splits > kMaxSplits) splits = kMaxSplits;
  // Normal (non-swap, single-CTA) tiles only: the collective phase needs the
  // whole grid resident (grid <= SMs) and the stage in row-major order.
  switch (cfg) {
    case kCfgP2N96: cfg = kCfgN96; break;
    case kCfgN192: case kCfgN96: case kCfgSwap128: case kCfgP2N128: case kCfgP2N192:
    case kCfgClN128: cfg = kCfgN128; break;
    case kCfgSwap16: case kCfgSwap32: case kCfgSwap64: case kCfgP2N64: cfg = kCfgN64; break;
    case kCfgM2N224: case kCfgM2N112: case kCfgClM2N128: case kCfgClM2N112: cfg = kCfgM2N128;
      break;
    case kCfgM2N64: case kCfgClM2N64: cfg = kCfgN64; break;
    case kCfgP2N256: cfg = kCfgM2N256; break;
    case kCfgClN256: cfg = kCfgN256; break;
    default: break;
  }
  const int num_kb = (K + 63) / 64;
  if (splits > num_kb) splits = num_kb;
  SplitWorkspace& sw = g_split_ws[dev];
  SplitGeometry geo = gemm_split_geometry(M, N, K, cfg, splits, num_sms(dev));
  if (splits > 1 && (sw.ws == nullptr || geo.ws_bytes > sw.ws_bytes || geo.counters > sw.n_counters))
    splits = 1;
  float* wsp = splits > 1 ? sw.ws : nullptr;
  int* cnt = splits > 1 ? sw.counters : nullptr;
  void* C = const_cast<__nv_bfloat16*>(ar.stage_peer[ar.rank]);
  WQParams wq{};
  wq.ar = ar;
#define B200_AR(BN_, ST_, MH_)                                                                \
  launch_cfg<BN_, ST_, false, kEpiArNorm, kWBf16, MH_>(A, W, C, M, N, K, lda, ldw, N, splits, \
                                                       wsp, cnt, err, stream, wq);            \
  return true
  switch (cfg) {
    case kCfgN256: B200_AR(256, 4, 1);
    case kCfgN64: B200_AR(64, 8, 1);
    case kCfgM2N256: B200_AR(256, 3, 2);
    case kCfgM2N128: B200_AR(128, 4, 2);
    default: B200_AR(128, 6, 1);
  }
#undef B200_AR
}

void gemm_wq_launch(const void* A, const void* Wraw, void* C, int M, int N, int K, int lda,
                    int ld_raw, int ldc, int wf, const WQParams& wq, int bn, int splits,
                    unsigned int* err, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return;
  if (K % 128 != 0) throw std::runtime_error("gemm_wq: K must be a multiple of 128");
  if (lda % 8 != 0 || ldc % 8 != 0 || N % 8 != 0)
    throw std::runtime_error("gemm_wq: leading dims / N must be multiples of 8");
  if (M > 256) throw std::runtime_error("gemm_wq: M > 256 uses dequantise + bf16 GEMM");
  int dev = 0;
  cudaGetDevice(&dev);
  const SplitWorkspace& w = g_split_ws[dev];
  if (bn <= 0) bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  const long tiles = (long)((N + 127) / 128) * ((M + bn - 1) / bn);
  const int num_kb = K / 64;
  if (splits <= 0) {
    splits = 1;
    const int sms = num_sms(dev);
    while (splits < kMaxSplits && tiles * (splits + 1) <= sms && num_kb / (splits + 1) >= 4)
      ++splits;
  }
  if (splits > 1) {
    const size_t need = (size_t)tiles * splits * 128 * bn * sizeof(float);
    if (w.ws == nullptr || need > w.ws_bytes || tiles > w.n_counters) splits = 1;
  }
  float* wsp = splits > 1 ? w.ws : nullptr;
  int* cnt = splits > 1 ? w.counters : nullptr;
#define B200_WQ(BN_, ST_, WF_)                                                                  \
  return (void)launch_cfg<BN_, ST_, true, kEpiNone, WF_>(Wraw, A, C, N, M, K, ld_raw, lda, ldc,   \
                                                         splits, wsp, cnt, err, stream, wq)
#define B200_WQ_BN(WF_)                          \
  switch (bn) {                                  \
    case 16: B200_WQ(16, 6, WF_);                \
    case 32: B200_WQ(32, 6, WF_);                \
    case 64: B200_WQ(64, 5, WF_);                \
    case 128: B200_WQ(128, 4, WF_);              \
    case 256: B200_WQ(256, 3, WF_);              \
    default: throw std::runtime_error("gemm_wq: bad BN"); \
  }
  switch (wf) {
    case kWFp8: B200_WQ_BN(kWFp8);
    case kWAwq: B200_WQ_BN(kWAwq);
    case kWNvfp4: B200_WQ_BN(kWNvfp4);
    default: throw std::runtime_error("gemm_wq: unknown weight format");
  }
#undef B200_WQ_BN
#undef B200_WQ
}

namespace {
// tile_off[e + 1] = tile_off[e] + (N / 128) * ceil(count_e / BN), on device.
__global__ void grouped_tiles_kernel(const int* __restrict__ row_off, int E, int nbs, int bn,
                                     int* __restrict__ tile_off) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int acc = 0;
  tile_off[0] = 0;
  for (int e = 0; e < E; ++e) {
    const int cnt = row_off[e + 1] - row_off[e];
    acc += nbs * ((cnt + bn - 1) / bn);
    tile_off[e + 1] = acc;
  }
}
}  // namespace

void gemm_grouped_launch(const void* X, const void* Wstk, void* C, int rows, int E, int N, int K,
                         int ldx, int ldw, int ldc, const int* row_off, int* tile_off, int wf,
                         const WQParams& wq, int bn, unsigned int* err, cudaStream_t stream) {
  if (rows <= 0 || E <= 0) return;
  if (N % 128 != 0) throw std::runtime_error("gemm_grouped: N per expert must be a multiple of 128");
  if (K % 64 != 0) throw std::runtime_error("gemm_grouped: K must be a multiple of 64");
  if (wf != kWBf16 && K % 128 != 0) throw std::runtime_error("gemm_grouped: quantised K % 128");
  if (bn <= 0) {
    const int avg = rows / E;
    bn = avg <= 16 ? 16 : avg <= 32 ? 32 : avg <= 64 ? 64 : avg <= 128 ? 128 : 256;
  }
  grouped_tiles_kernel<<<1, 32, 0, stream>>>(row_off, E, N / 128, bn, tile_off);
  GroupInfo g{tile_off, row_off, E, N};
  const int nbs = N / 128;
  const long max_tiles = (long)nbs * ((rows + bn - 1) / bn + E);
  const int units = (int)(max_tiles < (1 << 30) ? max_tiles : (1 << 30));
  const int P = E * N;
#define B200_G(BN_, ST_, WF_)                                                                   \
  return (void)launch_cfg<BN_, ST_, true, kEpiNone, WF_>(Wstk, X, C, P, rows, K, ldw, ldx, ldc, 1, \
                                                         nullptr, nullptr, err, stream, wq, g,   \
                                                         units)
#define B200_G_BN(WF_, S16, S64, S128, S256)                     \
  switch (bn) {                                                  \
    case 16: B200_G(16, S16, WF_);                               \
    case 32: B200_G(32, S16, WF_);                               \
    case 64: B200_G(64, S64, WF_);                               \
    case 128: B200_G(128, S128, WF_);                            \
    case 256: B200_G(256, S256, WF_);                            \
    default: throw std::runtime_error("gemm_grouped: bad BN");   \
  }
  switch (wf) {
    case kWBf16: B200_G_BN(kWBf16, 8, 8, 6, 4);
    case kWFp8: B200_G_BN(kWFp8, 6, 5, 4, 3);
    case kWAwq: B200_G_BN(kWAwq, 6, 5, 4, 3);
    case kWNvfp4: B200_G_BN(kWNvfp4, 6, 5, 4, 3);
    default: throw std::runtime_error("gemm_grouped: unknown weight format");
  }
#undef B200_G_BN
#undef B200_G
}

void gemm_bf16_launch(const void* A, const void* W, void* C, int M, int N, int K, int lda, int ldw,
                      int ldc, int epi, int cfg, unsigned int* err, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  const SplitWorkspace& w = g_split_ws[dev];
  gemm_bf16_launch_split(A, W, C, M, N, K, lda, ldw, ldc, epi, cfg, cfg < 0 ? 0 : 1, w.ws,
                         w.ws_bytes, w.counters, w.n_counters, err, stream, /*ext_reduce=*/true);
}

}  // namespace b200
