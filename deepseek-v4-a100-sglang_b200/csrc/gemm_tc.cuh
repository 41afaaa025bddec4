// MXFP4-weight x INT8-activation GEMM on the 5th-generation tensor core.
//
// One persistent kernel serves the dense GEMM (reference
// DENSE_ENTRY:334-433), the grouped MoE GEMMs W13 / W2 (reference
// MOE_ENTRY:146-272, MOE_CORE:380-646) and the W13 GEMM with a fused SwiGLU
// epilogue (reference PYMOE:916-935).
//
// Orientation ("swap-AB"): the decoded weight tile is the MMA A operand
// (M = 128 weight rows = output channels) and lives in tensor memory; the
// token rows are the B operand (N = 16..256 tokens, SW128 K-major
// in shared memory); int32 accumulators in TMEM, [channel lane][token col].
// One weight tile, once decoded, serves every token of the tile.
//
// Work items: (token block b, weight row tile y, K split z).  One CTA per SM
// walks items blockIdx.x, blockIdx.x + gridDim.x, ...; every role walks the
// same sequence, so the weight stream never drains between items.
//
// Issue cost shapes the design: in the issuing thread one tcgen05.mma costs
// ~70 cycles alone and ~100-200 beside ALU-bound decode warps, a completed
// mbarrier try_wait ~245 (so waits probe with test_wait first), one commit
// ~50.  So small token tiles spread the MMAs of alternate stages over 2-3
// issuer threads with their own accumulators (int32 sums are exact; the
// epilogue adds them), while 256-token tiles (N=256: 128 tensor cycles per
// MMA) need one.
//
// Warp roles (per token tile, see TcGemmCfg):
//   warp 0       TMA producer: packed FP4 codes, ONE tensor-map box per
//                256-K stage (gate and up halves in one 4-D box for SwiGLU),
//                and the 2-bit shifts of 32 stages in one box per chunk
//   warp 1       TMEM allocator; MMA issuer 0
//   warps 2..3   token rows of each stage into the SW128 B ring, and the
//                per-item metadata (rows, scales, channel scales by bulk copy).
//                Tiled modes: warp 2 metadata, warp 3 one 3-D box per stage
//                over K-chunk-major sorted rows (b_mode 2) or two 2-D boxes
//                over row-major rows (b_mode 1).  gather4 mode (b_mode 0):
//                both warps write metadata, then warp 2 + (g % 2) gathers the
//                rows of stage g with tile::gather4
//
// The per-SM TMA unit spends on the order of 100 cycles on every copy
// instruction however small, against ~750 cycles per stage at full HBM rate,
// so the number of copies per stage, not their bytes, is what is budgeted.
//   warps 4..    epilogue (4 warps, or 8 in two groups for 256-token tiles):
//                TMEM -> registers -> scales -> bf16 / int32 / SwiGLU ->
//                shared-memory staging -> 16-byte global stores
//   then         FP4 -> INT8 decode from the packed ring straight into TMEM
//                (tcgen05.st), kDecodeGroups groups of 4 warps, group g % G
//                takes stage g: one 64-column A slot per 128x256 stage
//   last warps   MMA issuers 1.. (issuer g % kIssuers takes stage g)
#pragma once

#include "common.cuh"

namespace dsv4 {

enum Epilogue : int { kEpiBf16 = 0, kEpiI32 = 1, kEpiSwiglu = 2 };
// Flag or-ed into the kernel's epilogue parameter: decode the weights to
// biased unsigned bytes (decode8_u8) and subtract 128 * a_rowsum[row] from
// every accumulator (needs per-row int8 sums over the item's K range, i.e.
// MoE items, which cover all of K).
constexpr int kEpiBiased = 4;
// Flag or-ed into the kernel's epilogue parameter: 256-token tiles on a CTA
// pair (cluster of 2, tcgen05.mma.cta_group::2, M = 256): each CTA decodes
// its own 128 weight rows and stages half of the token tile (tokens
// 128 r .. 128 r + 127 in CTA rank r), and the even CTA issues the MMAs for
// both.  Per SM a stage copies 48.5 KB instead of 80.5 KB.  Selected only
// with DSV4_B200_PAIR=1 (measured slower than single CTAs).
constexpr int kEpiPair = 8;

struct TcGemmParams {
  // Weight tensor maps (uint8):
  //   map_packed  3-D {128 B, NG8 groups, E*KB}: box {128, 16 (8 for SwiGLU), 4}
  //   map_shift   2-D {NG8*8 B, E*SS}:           box {128 (64 for SwiGLU), 1}
  //   SwiGLU: map_packed is 4-D {128 B, I/8 groups, 2 halves, E*KB}: box
  //   {128, 8, 2, 8}; map_shift is 3-D {I B, 2 halves, E*SS}: box {64, 2, R}
  //   (R = shift rows per chunk)
  CUtensorMap map_packed;
  CUtensorMap map_shift;
  // activations int8 [a_rows][lda] as 2-D {K, a_rows}, box {128 B, 1 row},
  // 128-byte swizzle: rows are gathered 4 at a time (tile::gather4)
  CUtensorMap map_act;
  // b_mode 2 on the sorted path: the same rows with a 64-row box, for blocks
  // whose sorted position 64 is already padding (short_rows = 64; 0: unused)
  CUtensorMap map_act_short;
  int short_rows;
  int kb_per_expert;        // KB = K / 32
  int ss_per_expert;        // shift stride SS
  // activations
  const int8_t* a;
  const float* a_scale;
  const int32_t* a_rowsum;  // biased decode: sum_k a[row][k], indexed like a_scale
  int64_t lda;
  int64_t a_rows;
  const float* cs;          // [E][N]
  int n;                    // weight rows (output channels) per expert
  int inter;                // SwiGLU: intermediate size (gate rows [0,I), up rows [I,2I))
  int k_stages;             // K / 128
  int stages_per_split;
  int splits;
  int row_tiles;            // weight row tiles per expert
  // token rows of each tile
  int moe;                  // 0: dense rows, 1: rows from the aligned permutation
  int m;                    // dense: number of rows
  int m_tiles;              // dense: number of token tiles
  const int32_t* sorted_ids;
  const int32_t* expert_ids;
  const int32_t* ntpp;      // num_tokens_post_padded[0]
  int block_m;
  int topk;
  int num_valid;
  int src_is_slot;
  int a_row_mode;           // MoE A rows / scales: 0 slot / topk, 1 slot, 2 sorted position
  int out_sorted;           // MoE output row: 0 slot, 1 sorted position
  int b_mode;               // 0 gather4, 1 2-D tile rows, 2 3-D K-chunk-major tile rows
  int sh_rows;              // shift rows per chunk box (2 per stage)
  // outputs
  __nv_bfloat16* out;
  int64_t ldo;
  int32_t* out_i32;
  int64_t split_stride;
  float clamp_limit;
  int has_clamp;
  // run-time constants of the decode (0xFFFFFFFF, 65536, 1): see decode8_fma
  uint32_t dec_m1;
  uint32_t dec_hi16;
  uint32_t dec_one;
};

// Ring discipline: an mbarrier parity wait is only safe if the waiter takes
// part in every use of that slot (otherwise it can run two phases ahead and
// see a stale phase as complete).  Every role therefore takes stage g by
// g mod (its count), and each ring depth is a multiple of those counts, so
// each slot always has the same waiter:
//   decode group  g % kDecodeGroups   -> kDecodeGroups | kStagesA, kStagesP
//   MMA issuer    g % kIssuers        -> kIssuers | kStagesA, kStagesB
//   gather warp   g % 2               -> 2 | kStagesB
//   token loader  waits for stage g - kStagesB on its A-slot empty barrier
//                 (safe while kStagesA >= kStagesB, see TcGemmCfg)
template <int TN, bool PAIR = false>
struct TcGemmCfg {
  static_assert(!PAIR || TN == 256, "CTA pairs run 256-token tiles");
  static constexpr int kBRows = PAIR ? TN / 2 : TN;  // token rows staged by this CTA
  static constexpr int kBHalf = kBRows * 128;    // one 128-K SW128 sub-tile of B
  static constexpr int kBBytes = 2 * kBHalf;     // kBRows token rows x 256 K (int8)
  static constexpr int kPBytes = 128 * 256 / 2;  // packed FP4 codes of one 256-K stage
  // shift chunks: the 2-bit shifts of kShChunk stages, [2 * kShChunk rows][128 B]
  // (row = one 4-block shift word per output row; SwiGLU: gate 64 B | up 64 B)
  static constexpr int kShChunk = TN >= 256 ? 16 : 32;  // (256-token tiles: smem is full)
  static constexpr int kShSlotBytes = 2 * kShChunk * 128;
  static constexpr int kShSlots = TN <= 64 ? 4 : 2;  // chunks in flight (short-K items: one each)
  static constexpr int kAccCols = TN;                     // N columns per accumulator
  // MMA issuer threads, one accumulator each: an issuer sharing its SM
  // sub-partition with three decode warps issues a 16-token MMA in ~200
  // cycles, so 16-token tiles (8 MMAs per stage) need three
  // (256-token tiles: an N=256 MMA takes 128 tensor cycles, more than its
  // issue cost, so one issuer keeps the tensor pipe busy)
  static constexpr int kIssuers = TN <= 16 ? 3 : (TN <= 128 ? 2 : 1);
  // groups of 4 decode warps (256-token tiles need a decoded stage per ~1000
  // cycles, which 8 warps deliver; their threads go to a second epilogue group)
  static constexpr int kDecodeGroups = TN <= 64 ? 3 : (TN <= 128 ? 4 : 2);
  // epilogue warps: 4, or 8 for 256-token tiles (two groups of 4 take
  // alternate 16-column chunks: that epilogue cannot overlap the next item's
  // MMAs, so its length counts in full)
  static constexpr int kEpiWarps = TN >= 192 ? 8 : 4;
  // A ring (decoded weights in TMEM, 64 columns = 256 K per slot) and B ring
  // (token tiles in shared memory) have their own depths and barriers
  // (192-token tiles: a 2-slot A ring leaves TMEM room for two accumulators,
  // so the next item's MMAs overlap the epilogue; 256-token tiles: a 2-slot
  // A ring leaves room for the epilogue's bf16 stash)
  static constexpr int kStagesA = TN <= 64 ? 6 : (TN >= 192 ? 2 : 4);
  // 256-token tiles (one accumulator of 256 columns): the epilogue first
  // converts the whole accumulator to bf16 pairs in a 128-column TMEM stash
  // and hands the accumulator back, then transposes and stores from the
  // stash while the next item's MMAs run
  static constexpr int kStashCols = TN == 256 ? 128 : 0;
  static constexpr int kStagesB = TN <= 64 ? 6 : (TN <= 128 ? 4 : 2);
  // One barrier pair per stage for both operands: the token-tile loader
  // arrives (with its bytes) on the A slot's ready barrier, and reuses B slot
  // g % kStagesB once the A-slot empty barrier shows stage g - kStagesB done.
  // Safe for parity waits because kStagesA >= kStagesB: when the loader waits
  // for stage g - kStagesB, every stage <= g - 1 - kStagesB is done already,
  // so the slot is never two phases behind, and the slot's previous ready
  // phase (stage g - kStagesA) has completed before the loader arrives.
  // accumulator sets per issuer: two where TMEM has room, so the MMAs of the
  // next item do not wait for the epilogue of this one
  static constexpr int kAccSlots =
      kIssuers * 2 * kAccCols + kStagesA * 64 + kStashCols <= 512 ? 2 : 1;
  // TMEM (512 columns): [issuer accumulators], [stash], then 64-column A slots
  static constexpr int kStashBase = kIssuers * kAccSlots * kAccCols;
  static constexpr int kAColBase = kStashBase + kStashCols;
  static constexpr int kTmemCols = 512;
  // epilogue staging, per epilogue group: 16 token columns x 128 rows bf16
  static constexpr int kStgBytes = (kEpiWarps / 4) * 16 * 128 * 2;
  // src, orow, ascale, rowsum [TN]; per-warp last [4]; channel scales [128]
  static constexpr int kMetaBytes = TN * 16 + 16 + 512;
  static constexpr int kMetaSlots = TN <= 128 ? 4 : 2;  // items of metadata prepared ahead
  static constexpr int kFixed = kStagesB * kBBytes + kShSlots * kShSlotBytes + kStgBytes + kMetaSlots * kMetaBytes + 1024;
  static constexpr int kBudget = 227 * 1024 - 1024;  // minus alignment slack
  static constexpr int kStagesPRaw = (kBudget - kFixed) / kPBytes;
  static constexpr int kStagesPCap = kStagesPRaw > 16 ? 16 : kStagesPRaw;
  static constexpr int kStagesP = kStagesPCap / kDecodeGroups * kDecodeGroups;
  static constexpr int kOffB = 0;
  static constexpr int kOffP = kOffB + kStagesB * kBBytes;
  static constexpr int kOffSh = kOffP + kStagesP * kPBytes;
  static constexpr int kOffStg = kOffSh + kShSlots * kShSlotBytes;
  static constexpr int kOffMeta = kOffStg + kStgBytes;
  static constexpr int kOffBar = kOffMeta + kMetaSlots * kMetaBytes;
  // barriers: pk_full/empty[SP], a_full/empty[SA], acc_full/empty[2],
  // meta_full/empty[kMetaSlots], sh_full/empty[kShSlots]
  static constexpr int kNumBars = 2 * kStagesP + 2 * kStagesA + 4 + 2 * kMetaSlots + 2 * kShSlots;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kSmemLaunch = kBytes + 1024;  // slack for 1024-B alignment
  // warps: 0 TMA, 1 issuer 0 + TMEM, 2-3 gather, epilogue, decode groups, issuers 1..
  static constexpr int kDecodeWarps = 4 * kDecodeGroups;
  static constexpr int kDecBase = 4 + kEpiWarps;
  static constexpr int kIssuer1Warp = kDecBase + kDecodeWarps;
  // idle warps so that issuers 1.. start on sub-partition 2 (issuer 0 is
  // warp 1, sub-partition 1): no sub-partition carries two issuers beside its
  // three ALU-bound decode warps (decode W2 -2 %)
  static constexpr int kIssuerPad = kIssuers > 1 ? (2 - kIssuer1Warp % 4 + 4) % 4 : 0;
  static constexpr int kWarps = kIssuer1Warp + kIssuerPad + kIssuers - 1;
  static constexpr int kThreads = kWarps * 32;
  static_assert(TN % 16 == 0 && TN >= 16 && TN <= 256, "token tile");
  static_assert(kStagesA % kDecodeGroups == 0 && kStagesA % kIssuers == 0 &&
                    kStagesB % kIssuers == 0 && kStagesB % 2 == 0 && kStagesA >= kStagesB,
                "ring discipline");
  static_assert(kStagesP % kDecodeGroups == 0 && kStagesP >= 3, "packed ring");
  static_assert(kAColBase + kStagesA * 64 <= kTmemCols, "TMEM budget");
  static_assert(kSmemLaunch <= 227 * 1024, "shared memory budget");
  static_assert(kBHalf % 1024 == 0 && kOffMeta % 16 == 0 && kOffBar % 8 == 0, "alignment");
};

__device__ __forceinline__ __nv_bfloat16 f2bf(float v) { return __float2bfloat16_rn(v); }

// SwiGLU tiles hold gate rows 0..63 and up rows 64..127 (channels j0..j0+63
// of each).  TMEM lane 32*quarter + lane carries gate row 16*quarter + lane
// (lane < 16) or up row 64 + 16*quarter + (lane - 16): the gate and up of a
// channel sit 16 lanes apart in the same warp.
__device__ __forceinline__ int swiglu_tile_row(int quarter, int lane) {
  return (lane < 16 ? 0 : 48) + 16 * quarter + lane;
}

struct Item {
  int b, y, z;
  int expert;
  bool valid;
};

// Item i of the persistent walk; `expert` is the expert id of its block
// (MoE), read ahead by ItemWalk.
__device__ __forceinline__ Item make_item(const TcGemmParams& p, int i, int expert) {
  Item it;
  if (p.moe) {
    // row tile fastest: CTAs running side by side stream neighbouring 2 KB
    // pieces of the same expert's K blocks
    it.z = 0;
    it.y = i % p.row_tiles;
    it.b = i / p.row_tiles;
    it.expert = expert;
    it.valid = it.expert >= 0;
  } else {
    it.z = i % p.splits;
    const int r = i / p.splits;
    it.b = r % p.m_tiles;
    it.y = r / p.m_tiles;
    it.expert = 0;
    it.valid = true;
  }
  return it;
}

// Every role walks items i0, i0 + G, ... (i0 = blockIdx.x, G = gridDim.x;
// CTA pairs: i0 = cluster index, G = number of clusters, and an item covers
// two neighbouring row tiles, CTA rank r taking row tile 2 y + r).  For MoE
// items the walk keeps (row tile, block) up to date by addition (no integer
// division by the run-time row-tile count at each item start: that chain of
// dependent instructions cost ~1,000 cycles of a decode warp per item) and
// reads the next item's expert id while the current item runs.
struct ItemWalk {
  const TcGemmParams& p;
  int n_items, G, rt, rank;  // rank: CTA rank in the pair, -1 without pairs
  int y, b, dy, db;          // MoE: coordinates of the next item; step per G
  int e_next;
  __device__ __forceinline__ ItemWalk(const TcGemmParams& p_, int n, int i0, int G_, int rank_)
      : p(p_), n_items(n), G(G_), rank(rank_) {
    rt = rank >= 0 ? p.row_tiles / 2 : p.row_tiles;
    y = i0 % rt;
    b = i0 / rt;
    dy = G % rt;
    db = G / rt;
    e_next = (p.moe && i0 < n_items) ? __ldg(p.expert_ids + b) : 0;
  }
  // item i (the walk's current one, in order); starts the read of the next
  __device__ __forceinline__ Item get(int i) {
    Item it;
    if (!p.moe) {
      it = make_item(p, i, 0);  // dense: pairs split row tiles as well
      if (rank >= 0) {
        const int r = i / p.splits;
        it.y = 2 * (r / p.m_tiles) + rank;
      }
      return it;
    }
    it.z = 0;
    it.y = rank >= 0 ? 2 * y + rank : y;
    it.b = b;
    it.expert = e_next;
    it.valid = it.expert >= 0;
    y += dy;
    b += db;
    if (y >= rt) {
      y -= rt;
      ++b;
    }
    e_next = (i + G < n_items) ? __ldg(p.expert_ids + b) : 0;
    return it;
  }
};

template <int TN, int EPIF>
__global__ void __launch_bounds__(TcGemmCfg<TN>::kThreads, 1)
mxfp4_int8_tc_gemm_kernel(const __grid_constant__ TcGemmParams p) {
  constexpr int EPI = EPIF & 3;
  constexpr bool kBiased = (EPIF & kEpiBiased) != 0;
  constexpr bool kPair = (EPIF & kEpiPair) != 0;
  using C = TcGemmCfg<TN, kPair>;
  constexpr int SA = C::kStagesA;
  constexpr int SB = C::kStagesB;
  constexpr int SP = C::kStagesP;
  constexpr int AS = C::kAccSlots;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  // Programmatic dependent launch: the next kernel may be scheduled now.  A
  // MoE GEMM waits for its predecessors here, before reading
  // num_tokens_post_padded; a dense GEMM sets up first (barriers, TMEM) and
  // its TMA weight producer never waits: the weights, shifts and tensor maps
  // are not written by the kernels it may overlap (the weight repack is an
  // ordinary launch, complete before any dependent starts), so its first
  // weight stages stream while the predecessor finishes.  Every other thread
  // waits before its first dependent access (activations, scales, outputs).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (p.moe) asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- the item space (identical in every thread; CTA pairs: in both CTAs) ----
  int n_blocks, n_items;
  const int row_items = kPair ? p.row_tiles / 2 : p.row_tiles;
  if (p.moe) {
    n_blocks = __ldg(p.ntpp) / p.block_m;
    n_items = n_blocks * row_items;
  } else {
    n_blocks = p.m_tiles;
    n_items = p.m_tiles * row_items * p.splits;
  }
  const int i_first = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int i_step = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int pair_rank = kPair ? static_cast<int>(cluster_ctarank()) : -1;
  if (i_first >= n_items) return;  // both CTAs of a pair leave together

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t bar0 = smem_u32(smem + C::kOffBar);
  auto pk_full = [&](int s) { return bar0 + 8u * s; };
  auto pk_empty = [&](int s) { return bar0 + 8u * (SP + s); };
  auto a_full = [&](int s) { return bar0 + 8u * (2 * SP + s); };
  auto a_empty = [&](int s) { return bar0 + 8u * (2 * SP + SA + s); };
  constexpr int kX = 2 * SP + 2 * SA;
  auto acc_full = [&](int s) { return bar0 + 8u * (kX + s); };
  auto acc_empty = [&](int s) { return bar0 + 8u * (kX + 2 + s); };
  constexpr int MS = C::kMetaSlots;
  auto meta_full = [&](int s) { return bar0 + 8u * (kX + 4 + s); };
  auto meta_empty = [&](int s) { return bar0 + 8u * (kX + 4 + MS + s); };
  constexpr int SHS = C::kShSlots;
  auto sh_full = [&](int s) { return bar0 + 8u * (kX + 4 + 2 * MS + s); };
  auto sh_empty = [&](int s) { return bar0 + 8u * (kX + 4 + 2 * MS + SHS + s); };
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  auto meta_src = [&](int s) {
    return reinterpret_cast<int*>(smem + C::kOffMeta + s * C::kMetaBytes);
  };
  auto meta_orow = [&](int s) { return meta_src(s) + TN; };
  auto meta_asc = [&](int s) { return reinterpret_cast<float*>(meta_src(s) + 2 * TN); };
  auto meta_rs = [&](int s) { return meta_src(s) + 3 * TN; };     // biased: -128 * rowsum
  auto meta_last = [&](int s) { return meta_src(s) + 4 * TN; };  // [2] per gather warp
  auto meta_cs = [&](int s) { return reinterpret_cast<float*>(meta_src(s) + 4 * TN + 4); };

  if (tid == 0) {
    for (int s = 0; s < SP; ++s) {
      mbar_init(pk_full(s), 1);
      mbar_init(pk_empty(s), 4);
    }
    // CTA pairs: the leader's a_full and acc_empty also count the peer's
    // arrivals (its decode group and token-tile lane, its epilogue warps)
    for (int s = 0; s < SA; ++s) {
      mbar_init(a_full(s), (kPair ? 2 : 1) * (4 + 1));  // decode group (4 warps) + token-tile lane
      mbar_init(a_empty(s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(acc_full(s), C::kIssuers);
      mbar_init(acc_empty(s), (kPair ? 2 : 1) * C::kEpiWarps);
    }
    for (int s = 0; s < SHS; ++s) {
      mbar_init(sh_full(s), 1);
      mbar_init(sh_empty(s), C::kDecodeWarps);
    }
    for (int s = 0; s < MS; ++s) {
      // metadata warps (two, or one in the tiled modes) + the channel-scale copy
      mbar_init(meta_full(s), p.b_mode != 0 ? 2 : 3);
      mbar_init(meta_empty(s), C::kEpiWarps);
    }
    mbar_fence_init();
  }
  if (warp == 1) {
    if constexpr (kPair) {
      tmem_alloc_pair(smem_u32(s_tmem), C::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(s_tmem), C::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  // CTA pairs: both CTAs' barriers are initialised before any remote arrival
  if constexpr (kPair) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  if (!p.moe && warp != 0) asm volatile("griddepcontrol.wait;" ::: "memory");
  // barriers that pair traffic goes to: the leader's (rank 0) copy
  auto leader = [&](uint32_t bar) { return kPair ? mapa_shared(bar, 0) : bar; };
  // arrivals on the leader's barriers: CTA scope from the leader's own
  // threads, cluster scope (remote) from the peer's
  auto arrive_leader = [&](uint32_t bar) {
    if (kPair && pair_rank != 0)
      mbar_arrive_cl(leader(bar));
    else
      mbar_arrive(bar);
  };
  // waits on barriers the peer arrives on, or (in the peer) that the
  // leader's pair commit signals, use cluster scope
  auto wait_x = [&](uint32_t bar, uint32_t parity, int code) {
    return kPair ? mbar_wait_cl(bar, parity, code) : mbar_wait(bar, parity, code);
  };
  auto wait_own = [&](uint32_t bar, uint32_t parity, int code) {
    return (kPair && pair_rank != 0) ? mbar_wait_cl(bar, parity, code)
                                     : mbar_wait(bar, parity, code);
  };

  // stages are 256 K (8 blocks of 32); the last one of K may be 128 K
  auto k_range = [&](const Item& it, int& ks0, int& nks) {
    ks0 = it.z * p.stages_per_split;
    nks = min(p.k_stages, ks0 + p.stages_per_split) - ks0;
  };
  auto stage_kb = [&](int ks) { return min(8, p.kb_per_expert - ks * 8); };
  auto n_mma_of = [&](int ms) {
    const int* lw = meta_last(ms);
    const int last = max(lw[0], lw[1]);
    return ((max(last, 0) + 16) / 16) * 16;
  };

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&p.map_packed);
      tma_prefetch_desc(&p.map_shift);
      const uint64_t pol = l2_policy_evict_first();
      const uint32_t sh_bytes = static_cast<uint32_t>(p.sh_rows) * 128u;
      uint32_t g = 0, cc = 0;
      ItemWalk walk(p, n_items, i_first, i_step, pair_rank);
      for (int i = i_first; i < n_items; i += i_step) {
        const Item it = walk.get(i);
        if (!it.valid) continue;
        int ks0, nks;
        k_range(it, ks0, nks);
        // SwiGLU: group g0 of the gate half (rows j0 .. j0+63; the up half is
        // the box's second plane); plain: rows 128*y .. 128*y+127
        const int g0 = EPI == kEpiSwiglu ? it.y * 8 : it.y * 16;
        for (int s = 0; s < nks; ++s, ++g) {
          const int ks = ks0 + s;
          if (s % C::kShChunk == 0) {
            // smem: [2 * kShChunk shift rows][128 B] (SwiGLU: gate 64 B | up 64 B)
            const int sl = cc % SHS;
            mbar_wait(sh_empty(sl), ((cc / SHS) & 1) ^ 1, kErrWaitPackedEmpty);
            mbar_arrive_expect_tx(sh_full(sl), sh_bytes);
            const uint32_t dsts = smem_u32(smem + C::kOffSh + sl * C::kShSlotBytes);
            const int sh_row = it.expert * p.ss_per_expert + ks * 2;
            if (EPI == kEpiSwiglu)
              tma_load_3d(dsts, &p.map_shift, it.y * 64, 0, sh_row, sh_full(sl), pol);
            else
              tma_load_2d(dsts, &p.map_shift, it.y * 128, sh_row, sh_full(sl), pol);
            ++cc;
          }
          const int sp = g % SP;
          mbar_wait(pk_empty(sp), ((g / SP) & 1) ^ 1, kErrWaitPackedEmpty);
          DSV4_TRACE_EV(0, g);
          mbar_arrive_expect_tx(pk_full(sp), C::kPBytes);
          const uint32_t dstp = smem_u32(smem + C::kOffP + sp * C::kPBytes);
          const int kb_row = it.expert * p.kb_per_expert + ks * 8;
          // smem: [kb 0..7][128 rows as 16 groups][128 B] (SwiGLU: gate groups
          // 0..7 then up groups 0..7 within each kb)
          if (EPI == kEpiSwiglu)
            tma_load_4d(dstp, &p.map_packed, 0, g0, 0, kb_row, pk_full(sp), pol);
          else
            tma_load_3d(dstp, &p.map_packed, 0, g0, kb_row, pk_full(sp), pol);
        }
      }
    }
  } else if (warp == 1 || warp >= C::kIssuer1Warp + C::kIssuerPad) {
    // ------------------------------- MMA issuers -------------------------------
    // takes stages g = j (mod kIssuers)
    const int j = warp == 1 ? 0 : warp - C::kIssuer1Warp - C::kIssuerPad + 1;
    // CTA pairs: the leader's issuer issues for both CTAs
    if (lane == 0 && j < C::kIssuers && pair_rank <= 0) {
      uint32_t g = 0, t = 0;
      const uint64_t bdesc0 = smem_desc_sw128(smem_u32(smem + C::kOffB));
      ItemWalk walk(p, n_items, i_first, i_step, pair_rank);
      for (int i = i_first; i < n_items; i += i_step) {
        const Item it = walk.get(i);
        if (!it.valid) continue;
        int ks0, nks;
        k_range(it, ks0, nks);
        const int ms = t % MS;
        const int as = t % AS;
        mbar_wait(meta_full(ms), (t / MS) & 1, kErrWaitMeta);
        // CTA pairs: M = 256 (128 rows per CTA) and always N = 256, split
        // 128 + 128 between the CTAs' token halves
        const int n_cols = kPair ? TN : n_mma_of(ms);
        const uint32_t m_rows = kPair ? 256u : 128u;
        const uint32_t idesc = kBiased ? idesc_u8s8(m_rows, n_cols) : idesc_i8(m_rows, n_cols);
        wait_x(acc_empty(as), ((t / AS) & 1) ^ 1, kErrWaitAccEmpty);
        if (j == 0) DSV4_TRACE_EV(12, t);
        tc_fence_after();
        const uint32_t d_tmem = tmem + (as * C::kIssuers + j) * C::kAccCols;
        const int s_first = static_cast<int>((j - static_cast<int>(g % C::kIssuers) + C::kIssuers) % C::kIssuers);
        for (int s = s_first; s < nks; s += C::kIssuers) {
          const uint32_t gs = g + s;
          const int sa = gs % SA;
          DSV4_TRACE_EV(9, gs);
          wait_x(a_full(sa), (gs / SA) & 1, kErrWaitAbFull);
          DSV4_TRACE_EV(3, gs);
          const uint32_t a_tmem = tmem + C::kAColBase + sa * 64;
          tc_fence_after();
          const int nkb = stage_kb(ks0 + s);
          const uint64_t bdesc = bdesc0 + static_cast<uint64_t>(((gs % SB) * C::kBBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            if (kk < nkb) {
              const uint64_t bd =
                  bdesc + static_cast<uint64_t>(((kk >> 2) * C::kBHalf + (kk & 3) * 32) >> 4);
              const uint32_t acc = (s > s_first || kk > 0) ? 1u : 0u;
              if constexpr (kPair)
                mma_i8_ts_pair(d_tmem, a_tmem + kk * 8, bd, idesc, acc);
              else
                mma_i8_ts(d_tmem, a_tmem + kk * 8, bd, idesc, acc);
            }
          }
          // frees the A slot and (for the loader) the B slot; pairs: in both CTAs
          if constexpr (kPair) {
            mma_commit_pair(mapa_shared(a_empty(sa), 0));
            mma_commit_pair(mapa_shared(a_empty(sa), 1));
          } else {
            mma_commit(a_empty(sa));
          }
          DSV4_TRACE_EV(6, gs);
        }
        if constexpr (kPair) {
          mma_commit_pair(mapa_shared(acc_full(as), 0));
          mma_commit_pair(mapa_shared(acc_full(as), 1));
        } else {
          mma_commit(acc_full(as));
        }
        g += nks;
        ++t;
      }
    }
  } else if (warp < 4) {
    // ------------------- token metadata + activation tiles -------------------
    // Tiled modes (b_mode 1, 2): warp 2 writes the metadata of every item and
    // warp 3 loads the token tile of every stage (it needs only the block's
    // first row, so it never waits for metadata).  gather4 mode (b_mode 0):
    // both warps write the metadata, then take alternate stages, gathering
    // the rows the metadata names.
    const bool tiled = p.b_mode != 0;
    const uint64_t pol = l2_policy_evict_last();  // token rows are re-read by every row tile
    if (tiled && warp == 3) {
      if (lane == 0) {
        tma_prefetch_desc(&p.map_act);
        // A block whose sorted position short_rows holds padding has at most
        // short_rows tokens (padding ends an expert's last block): its stages
        // copy a short_rows-row box (the MMAs read only the block's columns).
        // The test of the next item is read while the current one loads.
        const bool use_short = !kPair && p.moe && p.b_mode == 2 && p.short_rows > 0;
        if (use_short) tma_prefetch_desc(&p.map_act_short);
        auto is_short = [&](int b) {
          return __ldg(p.sorted_ids + static_cast<int64_t>(b) * p.block_m + p.short_rows) >=
                 p.num_valid;
        };
        uint32_t g = 0;
        ItemWalk walk(p, n_items, i_first, i_step, pair_rank);
        bool short_next = use_short && i_first < n_items ? is_short(walk.b) : false;
        for (int i = i_first; i < n_items; i += i_step) {
          const Item it = walk.get(i);
          const bool shrt = short_next;
          short_next = use_short && i + i_step < n_items ? is_short(walk.b) : false;
          if (!it.valid) continue;
          int ks0, nks;
          k_range(it, ks0, nks);
          const int row0 = p.moe ? it.b * p.block_m : it.b * TN;
          for (int s = 0; s < nks; ++s, ++g) {
            const int sb = g % SB;
            const uint32_t ready = a_full(g % SA);
            if (g >= static_cast<uint32_t>(SB))  // B slot free once stage g - SB is done
              wait_own(a_empty((g - SB) % SA), ((g - SB) / SA) & 1, kErrWaitAbEmpty);
            DSV4_TRACE_EV(7, g);
            const uint32_t b_base = smem_u32(smem + C::kOffB + sb * C::kBBytes);
            if (kPair) {
              // this CTA's half of the token tile, completing on the leader's barrier
              const uint32_t rdy = leader(ready);
              if (pair_rank != 0)
                mbar_arrive_expect_tx_cl(rdy, static_cast<uint32_t>(C::kBBytes));
              else
                mbar_arrive_expect_tx(ready, static_cast<uint32_t>(C::kBBytes));
              tma_load_3d_pair(b_base, &p.map_act, 0, row0 + pair_rank * C::kBRows,
                               (ks0 + s) * 2, rdy, pol);
            } else if (p.b_mode == 2) {
              // [K/128][rows][128]: one box {128, TN, 2} = both 128-K halves;
              // short blocks: a {128, short_rows, 1} box into each half (the
              // MMA descriptors address the second half kBHalf bytes on)
              if (shrt) {
                mbar_arrive_expect_tx(ready, static_cast<uint32_t>(p.short_rows) * 256u);
                tma_load_3d(b_base, &p.map_act_short, 0, row0, (ks0 + s) * 2, ready, pol);
                tma_load_3d(b_base + C::kBHalf, &p.map_act_short, 0, row0, (ks0 + s) * 2 + 1,
                            ready, pol);
              } else {
                mbar_arrive_expect_tx(ready, static_cast<uint32_t>(C::kBBytes));
                tma_load_3d(b_base, &p.map_act, 0, row0, (ks0 + s) * 2, ready, pol);
              }
            } else {
              const int nhalf = stage_kb(ks0 + s) > 4 ? 2 : 1;
              mbar_arrive_expect_tx(ready, static_cast<uint32_t>(nhalf * C::kBHalf));
              tma_load_2d(b_base, &p.map_act, (ks0 + s) * 256, row0, ready, pol);
              if (nhalf == 2)
                tma_load_2d(b_base + C::kBHalf, &p.map_act, (ks0 + s) * 256 + 128, row0,
                            ready, pol);
            }
            DSV4_TRACE_EV(4, g);
          }
        }
      }
    } else {
      const int nthr = tiled ? 32 : 64;
      const int gt = tid - 64;  // < nthr
      uint32_t g = 0, t = 0;
      if (gt == 0 && !tiled) tma_prefetch_desc(&p.map_act);
      ItemWalk walk(p, n_items, i_first, i_step, pair_rank);
      for (int i = i_first; i < n_items; i += i_step) {
        const Item it = walk.get(i);
        if (!it.valid) continue;
        int ks0, nks;
        k_range(it, ks0, nks);
        const int ms = t % MS;
        mbar_wait(meta_empty(ms), ((t / MS) & 1) ^ 1, kErrWaitMeta);
        if (gt == 0) {
          // channel scales of the item's 128 weight rows, copied into the
          // metadata slot (a cold load in the epilogue costs microseconds)
          if (EPI == kEpiI32) {
            mbar_arrive(meta_full(ms));
          } else {
            const float* cs_e = p.cs + static_cast<int64_t>(it.expert) * p.n;
            const uint32_t dcs = smem_u32(meta_cs(ms));
            mbar_arrive_expect_tx(meta_full(ms), 512);
            if (EPI == kEpiSwiglu) {
              bulk_g2s(dcs, cs_e + it.y * 64, 256, meta_full(ms), pol);
              bulk_g2s(dcs + 256, cs_e + p.inter + it.y * 64, 256, meta_full(ms), pol);
            } else {
              bulk_g2s(dcs, cs_e + it.y * 128, 512, meta_full(ms), pol);
            }
          }
        }
        int* src_s = meta_src(ms);
        int* orow_s = meta_orow(ms);
        float* asc_s = meta_asc(ms);
        int* rs_s = meta_rs(ms);
        const bool by_pos = p.moe && p.a_row_mode == 2;
        int my_last = -1;
        for (int jj = gt; jj < TN; jj += nthr) {
          int src = -1, orow = -1;
          float asc = 0.f;
          int rs = 0;
          if (p.moe) {
            if (jj < p.block_m) {
              const int pos = it.b * p.block_m + jj;
              // sorted rows: scale and row sum are indexed by position, so
              // their loads need not wait for the slot id
              float asc_pos = 0.f;
              int rs_pos = 0;
              if (by_pos) {
                asc_pos = __ldg(p.a_scale + pos);
                if (kBiased) rs_pos = __ldg(p.a_rowsum + pos);
              }
              const int slot = __ldg(p.sorted_ids + pos);
              if (slot >= 0 && slot < p.num_valid) {
                src = by_pos ? pos : (p.a_row_mode == 1 ? slot : slot / p.topk);
                orow = p.out_sorted ? pos : slot;
                asc = asc_pos;
                rs = rs_pos;
              }
            }
          } else {
            const int m = it.b * TN + jj;
            if (m < p.m) src = orow = m;
          }
          if (src >= p.a_rows) src = -1, orow = -1;
          if (src >= 0) {
            if (!by_pos) {
              asc = p.a_scale != nullptr ? __ldg(p.a_scale + src) : 0.f;
              if (kBiased) rs = __ldg(p.a_rowsum + src);
            }
            my_last = jj;
          }
          src_s[jj] = src;
          orow_s[jj] = orow;
          asc_s[jj] = asc;
          if (kBiased) rs_s[jj] = src >= 0 ? -128 * rs : 0;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
          my_last = max(my_last, __shfl_xor_sync(0xffffffffu, my_last, o));
        if (lane == 0) {
          meta_last(ms)[warp - 2] = my_last;
          if (tiled) meta_last(ms)[1] = -1;
        }
        if (tiled)
          __syncwarp();
        else
          named_bar_sync(2, 64);
        __syncwarp();
        if (lane == 0) mbar_arrive(meta_full(ms));
        if (!tiled) {
          // Warps 2 and 3 take alternate stages and gather only the rows up to
          // the last valid one (4 at a time, lane l -> rows 4l .. 4l+3 of both
          // 128-K halves); the MMA columns beyond are never stored.
          const int last = max(meta_last(ms)[0], meta_last(ms)[1]);
          const int n_rows = ((max(last, 0) + 4) / 4) * 4;
          for (int s = 0; s < nks; ++s, ++g) {
            if (static_cast<int>(g & 1) != warp - 2) continue;
            const int sb = g % SB;
            const uint32_t ready = a_full(g % SA);
            const int nhalf = stage_kb(ks0 + s) > 4 ? 2 : 1;
            if (lane == 0) {
              if (g >= static_cast<uint32_t>(SB))  // B slot free once stage g - SB is done
                mbar_wait(a_empty((g - SB) % SA), ((g - SB) / SA) & 1, kErrWaitAbEmpty);
              DSV4_TRACE_EV(7, g);
              mbar_arrive_expect_tx(ready, static_cast<uint32_t>(nhalf * n_rows * 128));
            }
            __syncwarp();
            const int x0 = (ks0 + s) * 256;
            const uint32_t b_base = smem_u32(smem + C::kOffB + sb * C::kBBytes);
            for (int r = lane * 4; r < n_rows; r += 128) {
              const uint32_t dst = b_base + (r >> 3) * 1024 + (r & 7) * 128;
              // padding rows read the out-of-range row -1: zeros
              tma_gather4(dst, &p.map_act, x0, src_s[r], src_s[r + 1], src_s[r + 2],
                          src_s[r + 3], ready, pol);
              if (nhalf == 2)
                tma_gather4(dst + C::kBHalf, &p.map_act, x0 + 128, src_s[r], src_s[r + 1],
                            src_s[r + 2], src_s[r + 3], ready, pol);
            }
            if (lane == 0) DSV4_TRACE_EV(4, g);
          }
        }
        ++t;
      }
    }
  } else if (warp < C::kDecBase) {
    // -------------------------------- epilogue --------------------------------
    constexpr int EH = C::kEpiWarps / 4;  // epilogue groups: group eh takes chunks eh, eh + EH, ..
    const int eh = (warp - 4) >> 2;
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    const int row_local = quarter * 32 + lane;
    // weight row (within the tile) held in this thread's TMEM lane: SwiGLU
    // tiles put the gate and up rows of a channel in one warp
    // (swiglu_tile_row), so the pairing is a shuffle
    const int wrow = EPI == kEpiSwiglu ? swiglu_tile_row(quarter, lane) : row_local;
    // this warp's private staging slice (1 KB): the transpose of a 16-token
    // chunk goes through it with __syncwarp only, no barrier between warps
    uint16_t* stw = reinterpret_cast<uint16_t*>(smem + C::kOffStg + (warp - 4) * 1024);
    const float lim = p.has_clamp ? __bfloat162float(f2bf(p.clamp_limit)) : 0.f;
    uint32_t t = 0, g = 0;
    ItemWalk walk(p, n_items, i_first, i_step, pair_rank);
    for (int i = i_first; i < n_items; i += i_step) {
      const Item it = walk.get(i);
      if (!it.valid) continue;
      int ks0, nks;
      k_range(it, ks0, nks);
      const int ms = t % MS;
      const int as = t % AS;
      mbar_wait(meta_full(ms), (t / MS) & 1, kErrWaitMeta);
      wait_own(acc_full(as), (t / AS) & 1, kErrWaitAccFull);
      if (tid == 128) DSV4_TRACE_EV(10, t);
      tc_fence_after();
      const int* orow_s = meta_orow(ms);
      const float* asc_s = meta_asc(ms);
      const int* rs_s = meta_rs(ms);
      const int n_mma = n_mma_of(ms);
      // accumulators written: issuers (g + s) % kIssuers for s < nks
      uint32_t accmask = 0;
      for (int q = 0; q < min(nks, C::kIssuers); ++q) accmask |= 1u << ((g + q) % C::kIssuers);
      const uint32_t t0 = tmem + (as * C::kIssuers) * C::kAccCols + (static_cast<uint32_t>(quarter * 32) << 16);
      const float csn = EPI == kEpiI32 ? 0.f : meta_cs(ms)[wrow];
      // One accumulator (kIssuers == 1, the 256-token tiles): the TMEM load of
      // the next 16 columns is issued before this chunk is processed, so its
      // latency overlaps the chunk's work.
      int32_t pre[16];
      // stash tiles load the accumulator 32 columns at a time (their own loop)
      constexpr bool kX32 = C::kStashCols > 0 && EPI != kEpiI32;
      if constexpr (C::kIssuers == 1 && !kX32) tmem_ld_x16(t0 + 16 * eh, pre);
      bool acc_released = false;
      auto release_acc = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) arrive_leader(acc_empty(as));
        acc_released = true;
      };
      auto load16 = [&](int c0, int32_t (&v)[16]) {
        if (kBiased) {  // row-sum corrections of the 16 tokens, 4 vector loads
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const int4 r = reinterpret_cast<const int4*>(rs_s + c0)[q4];
            v[4 * q4] = r.x, v[4 * q4 + 1] = r.y, v[4 * q4 + 2] = r.z, v[4 * q4 + 3] = r.w;
          }
        } else {
#pragma unroll
          for (int q = 0; q < 16; ++q) v[q] = 0;
        }
        if constexpr (C::kIssuers == 1) {
          tmem_ld_wait_regs(pre);
#pragma unroll
          for (int q = 0; q < 16; ++q) v[q] += pre[q];
          if (c0 + 16 * EH < n_mma) tmem_ld_x16(t0 + c0 + 16 * EH, pre);
        } else {
          for (int a = 0; a < C::kIssuers; ++a) {
            if (!(accmask & (1u << a))) continue;
            int32_t w[16];
            tmem_ld_x16(t0 + a * C::kAccCols + c0, w);
            tmem_ld_wait();
#pragma unroll
            for (int q = 0; q < 16; ++q) v[q] += w[q];
          }
        }
        // One accumulator (no second slot to run ahead into): after this
        // warp's last chunk load its TMEM reads are complete, so the
        // accumulator is handed back now and the next item's MMAs overlap
        // the chunk's scaling and stores.
        if (C::kIssuers == 1 && c0 + 16 * EH >= n_mma) release_acc();
      };

      // bf16((f32(acc) * a_scale) * cs) of the 16 tokens of a chunk, in the
      // reference order, two values rounded per conversion (the same
      // round-to-nearest-even per value)
      auto scale16 = [&](int c0, const int32_t (&v)[16], uint32_t (&pk)[8]) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const float4 a = reinterpret_cast<const float4*>(asc_s + c0)[q4];
          const float x0 = __fmul_rn(__fmul_rn(__int2float_rn(v[4 * q4]), a.x), csn);
          const float x1 = __fmul_rn(__fmul_rn(__int2float_rn(v[4 * q4 + 1]), a.y), csn);
          const float x2 = __fmul_rn(__fmul_rn(__int2float_rn(v[4 * q4 + 2]), a.z), csn);
          const float x3 = __fmul_rn(__fmul_rn(__int2float_rn(v[4 * q4 + 3]), a.w), csn);
          const __nv_bfloat162 p01 = __floats2bfloat162_rn(x0, x1);
          const __nv_bfloat162 p23 = __floats2bfloat162_rn(x2, x3);
          pk[2 * q4] = *reinterpret_cast<const uint32_t*>(&p01);
          pk[2 * q4 + 1] = *reinterpret_cast<const uint32_t*>(&p23);
        }
      };

      // the chunk's output from its 16 scaled bf16 values (pk[p]: tokens 2p, 2p+1)
      auto emit16 = [&](int c0, const uint32_t (&pk)[8]) {
        if constexpr (EPI == kEpiSwiglu) {
          // lanes 0..15: gate of channels j0 + 16*quarter + (lane & 15); lanes
          // 16..31: up of the same channels.  Gate lanes finish tokens 0..7,
          // up lanes tokens 8..15, after swapping the other half by shuffle.
          const int j0 = it.y * 64;
          const bool is_gate = lane < 16;
          const int chl = lane & 15;
          uint32_t mine[4], other[4];
#pragma unroll
          for (int pp = 0; pp < 4; ++pp) {
            const uint32_t send = is_gate ? pk[4 + pp] : pk[pp];  // gate: tokens 8..15, up: 0..7
            other[pp] = __shfl_xor_sync(0xffffffffu, send, 16);
            mine[pp] = is_gate ? pk[pp] : pk[4 + pp];
          }
          const int tok0 = is_gate ? 0 : 8;
          uint32_t hw[4];
#pragma unroll
          for (int pp = 0; pp < 4; ++pp) {
            const uint32_t gw = is_gate ? mine[pp] : other[pp];
            const uint32_t uw = is_gate ? other[pp] : mine[pp];
            float2 gv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw));
            float2 up = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&uw));
            if (p.has_clamp) {
              gv.x = fminf(gv.x, lim), gv.y = fminf(gv.y, lim);
              up.x = fminf(fmaxf(up.x, -lim), lim), up.y = fminf(fmaxf(up.y, -lim), lim);
            }
            // silu in fast fp32 (MUFU exp2 / reciprocal): the result is
            // rounded to bf16, where it differs from the IEEE-exact form by
            // at most one ulp, and rarely
            const float2 sg = __bfloat1622float2(
                __floats2bfloat162_rn(__fdividef(gv.x, 1.0f + __expf(-gv.x)),
                                      __fdividef(gv.y, 1.0f + __expf(-gv.y))));
            const __nv_bfloat162 hh =
                __floats2bfloat162_rn(__fmul_rn(sg.x, up.x), __fmul_rn(sg.y, up.y));
            hw[pp] = *reinterpret_cast<const uint32_t*>(&hh);
          }
          // staging [16 tokens][16 channels] bf16 as 32-bit words of two
          // channels: lanes (2j, 2j+1) of a half swap token halves by
          // shuffle; the even lane writes tokens tok0 + 0..3, the odd lane
          // tok0 + 4..7 of channels (2j, 2j+1), each of the four lane groups
          // starting at a different row so one store spans all banks
          {
            const uint32_t odd = chl & 1;
            const uint32_t r0 = __shfl_xor_sync(0xffffffffu, odd ? hw[0] : hw[2], 1);
            const uint32_t r1 = __shfl_xor_sync(0xffffffffu, odd ? hw[1] : hw[3], 1);
            const uint32_t o0 = odd ? hw[2] : hw[0], o1 = odd ? hw[3] : hw[1];
            const uint32_t e0 = odd ? r0 : o0, d0 = odd ? o0 : r0;
            const uint32_t e1 = odd ? r1 : o1, d1 = odd ? o1 : r1;
            uint32_t wv4[4];
            wv4[0] = (e0 & 0xFFFFu) | (d0 << 16);
            wv4[1] = (e0 >> 16) | (d0 & 0xFFFF0000u);
            wv4[2] = (e1 & 0xFFFFu) | (d1 << 16);
            wv4[3] = (e1 >> 16) | (d1 & 0xFFFF0000u);
            const int tb = tok0 + (odd ? 4 : 0);
            const int gidx = (lane >> 4) * 2 + static_cast<int>(odd);
            uint32_t* s32 = reinterpret_cast<uint32_t*>(stw);
#pragma unroll
            for (int x = 0; x < 4; ++x) {
              const int xx = (x + gidx) & 3;
              uint32_t val = wv4[0];
              val = xx == 1 ? wv4[1] : val;
              val = xx == 2 ? wv4[2] : val;
              val = xx == 3 ? wv4[3] : val;
              s32[(tb + xx) * 8 + (chl >> 1)] = val;
            }
          }
          __syncwarp();
          {
            const int tok = lane >> 1, half = lane & 1;
            const int orow = orow_s[c0 + tok];
            const uint4 hq = *reinterpret_cast<const uint4*>(stw + tok * 16 + 8 * half);
            if (orow >= 0)
              *reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(orow) * p.ldo + j0 +
                                        16 * quarter + 8 * half) = hq;
          }
          __syncwarp();
        } else {
          // transpose through the warp's staging slice [16 tokens][32
          // channels]: lane 8a + i then stores channels 8a..8a+7 of tokens
          // i and 8 + i as two 16-byte stores (each token row of the warp
          // is 64 contiguous bytes).  32-bit words of two neighbouring
          // channels: lane pairs (2j, 2j+1) swap halves by shuffle, the even
          // lane then writes tokens 0..7 and the odd lane tokens 8..15 of
          // channels (2j, 2j+1); rows of opposite parity in one store keep
          // the two lane sets on different banks
          {
            const uint32_t odd = lane & 1;
            const int tb = odd ? 8 : 0, j = lane >> 1;
            uint32_t* s32 = reinterpret_cast<uint32_t*>(stw);
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
              const uint32_t par = __shfl_xor_sync(0xffffffffu, odd ? pk[qq] : pk[4 + qq], 1);
              const uint32_t own = odd ? pk[4 + qq] : pk[qq];
              const uint32_t ev = odd ? par : own, od = odd ? own : par;
              const uint32_t w0 = (ev & 0xFFFFu) | (od << 16);          // token tb + 2qq
              const uint32_t w1 = (ev >> 16) | (od & 0xFFFF0000u);      // token tb + 2qq + 1
              s32[(tb + 2 * qq + odd) * 16 + j] = odd ? w1 : w0;
              s32[(tb + 2 * qq + 1 - odd) * 16 + j] = odd ? w0 : w1;
            }
          }
          __syncwarp();
          const int i = lane & 7, a8 = (lane >> 3) * 8;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int tok = 8 * h + i;
            const int orow = orow_s[c0 + tok];
            const uint4 val = *reinterpret_cast<const uint4*>(stw + tok * 32 + a8);
            if (orow >= 0)
              *reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(orow) * p.ldo +
                                        it.y * 128 + quarter * 32 + a8) = val;
          }
          __syncwarp();
        }
      };

      if constexpr (EPI == kEpiI32) {
        const int n_g = it.y * 128 + row_local;
        for (int c0 = 16 * eh; c0 < n_mma; c0 += 16 * EH) {
          int32_t v[16];
          load16(c0, v);
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const int orow = orow_s[c0 + q];
            if (orow < 0) continue;
            p.out_i32[static_cast<int64_t>(it.z) * p.split_stride +
                      static_cast<int64_t>(orow) * p.ldo + n_g] = v[q];
          }
        }
      } else if constexpr (kX32) {
        // Stash tiles (256 tokens, one accumulator).  Phase 1: the whole
        // accumulator -> scaled bf16 pairs in the TMEM stash (8 columns per
        // 16-token chunk), 32 accumulator columns per load (group eh owns
        // 32-column blocks eh, eh + EH, .. in both phases); the accumulator
        // goes back after the warp's last load, so the next item's MMAs
        // start while phase 2 transposes and stores from the stash.
        const uint32_t st0 = tmem + C::kStashBase + (static_cast<uint32_t>(quarter * 32) << 16);
        for (int b0 = 32 * eh; b0 < n_mma; b0 += 32 * EH) {
          int32_t w[32];
          tmem_ld_x32_wait(t0 + b0, w);
          if (b0 + 32 * EH >= n_mma) release_acc();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c0 = b0 + 16 * h;
            if (c0 < n_mma) {
              int32_t v[16];
              if (kBiased) {
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                  const int4 r = reinterpret_cast<const int4*>(rs_s + c0)[q4];
                  v[4 * q4] = r.x + w[16 * h + 4 * q4];
                  v[4 * q4 + 1] = r.y + w[16 * h + 4 * q4 + 1];
                  v[4 * q4 + 2] = r.z + w[16 * h + 4 * q4 + 2];
                  v[4 * q4 + 3] = r.w + w[16 * h + 4 * q4 + 3];
                }
              } else {
#pragma unroll
                for (int q = 0; q < 16; ++q) v[q] = w[16 * h + q];
              }
              uint32_t pk[8];
              scale16(c0, v, pk);
              tmem_st_x8(st0 + c0 / 2, pk);
            }
          }
        }
        tmem_st_wait();
        for (int b0 = 32 * eh; b0 < n_mma; b0 += 32 * EH) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c0 = b0 + 16 * h;
            if (c0 < n_mma) {
              uint32_t pk[8];
              tmem_ld_x8(st0 + c0 / 2, pk);
              tmem_ld_wait_regs8(pk);
              emit16(c0, pk);
            }
          }
        }
      } else {
        for (int c0 = 16 * eh; c0 < n_mma; c0 += 16 * EH) {
          int32_t v[16];
          load16(c0, v);
          uint32_t pk[8];
          scale16(c0, v, pk);
          emit16(c0, pk);
        }
      }
      if (!acc_released) {  // a group with no chunk of this item
        if constexpr (C::kIssuers == 1) tmem_ld_wait_regs(pre);
        release_acc();
      }
      __syncwarp();
      if (tid == 128) DSV4_TRACE_EV(11, t);
      if (lane == 0) mbar_arrive(meta_empty(ms));
      g += nks;
      ++t;
    }
  } else if (warp < C::kIssuer1Warp) {
    // ------------------------- FP4 -> INT8 decode -> TMEM -------------------------
    // kDecodeGroups groups of 4 warps; group g % G takes stage g; in a group warp w covers TMEM
    // lane quarter w % 4 (rows 32*(w%4) ..) and all 8 32-K blocks of the stage
    // (64 TMEM columns: block kb -> columns 8kb .. 8kb+7).
    const int quarter = warp & 3;
    const int grp = (warp - C::kDecBase) >> 2;
    // weight row of the tile decoded into this thread's TMEM lane
    const int row = EPI == kEpiSwiglu ? swiglu_tile_row(quarter, lane) : quarter * 32 + lane;
    const uint32_t t_lane = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t m1 = p.dec_m1, hi16 = p.dec_hi16, one = p.dec_one;
    uint32_t g = 0, cc = 0;
    // MoE items all cover the whole K range, so their stage count is fixed
    // and this group's first stage in the next item follows by a subtraction
    // (the item start is a serial chain of control instructions on a busy
    // sub-partition: every instruction taken out of it shortens the gap)
    const int G = C::kDecodeGroups;
    const int nks_moe = p.k_stages, nks_mod = p.k_stages % G;
    int s_first = grp;  // g = 0
    ItemWalk walk(p, n_items, i_first, i_step, pair_rank);
    for (int i = i_first; i < n_items; i += i_step) {
      const Item it = walk.get(i);
      if (!it.valid) continue;
      int ks0 = 0, nks = nks_moe;
      if (!p.moe) k_range(it, ks0, nks);
      // Only this group's stages are visited (s = s_first, s_first + G, ...):
      // stepping through the other groups' stages cost hundreds of cycles
      // each.  Every decode warp still takes part in every shift chunk (ring
      // discipline), whether or not it has a stage in it.
      int s = p.moe ? s_first
                    : static_cast<int>((grp - static_cast<int>(g % G) + G) % G);
      for (int c0 = 0; c0 < nks; c0 += C::kShChunk, ++cc) {
        mbar_wait(sh_full(cc % SHS), (cc / SHS) & 1, kErrWaitPackedFull);
        const uint8_t* SHC = smem + C::kOffSh + (cc % SHS) * C::kShSlotBytes;
        const int c1 = min(nks, c0 + C::kShChunk);
        for (; s < c1; s += C::kDecodeGroups) {
          const uint32_t gs = g + static_cast<uint32_t>(s);
          const int sp = gs % SP;
          const int sa = gs % SA;
          const int nkb = stage_kb(ks0 + s);
          if (lane == 0 && quarter == 0) DSV4_TRACE_EV(8, gs);
          mbar_wait(pk_full(sp), (gs / SP) & 1, kErrWaitPackedFull);
          if (lane == 0 && quarter == 0) DSV4_TRACE_EV(1, gs);
          const uint8_t* P = smem + C::kOffP + sp * C::kPBytes;
          const uint8_t* SH = SHC + (s % C::kShChunk) * 256;
          uint32_t shw[2];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) shw[hh] = SH[hh * 128 + row];
          // decode of 8 weights (biased unsigned on the sorted path)
          auto dec8 = [&](uint32_t q, uint32_t a0, uint32_t a1, uint32_t& lo, uint32_t& hi) {
            if (kBiased) decode8_u8(q, a0, a1, one, m1, hi16, lo, hi);
            else decode8_fma(q, a0, a1, m1, hi16, lo, hi);
          };
          // all 8 packed units first (a 128-K tail stage decodes stale bytes
          // into columns the MMA never reads)
          uint4 wv[8];
#pragma unroll
          for (int kb = 0; kb < 8; ++kb) {
            const int poff = kb * 2048 + row * 16;
            wv[kb] = *reinterpret_cast<const uint4*>(P + poff);
          }
          (void)nkb;
          wait_own(a_empty(sa), ((gs / SA) & 1) ^ 1, kErrWaitAbEmpty);
          if (lane == 0 && quarter == 0) DSV4_TRACE_EV(2, gs);
          tc_fence_after();
          const uint32_t tcol = tmem + t_lane + C::kAColBase + sa * 64;
#pragma unroll
          for (int q = 0; q < 4; ++q) {  // blocks 2q, 2q+1 -> columns 16q .. 16q+15
            uint32_t v[16];
#pragma unroll
            for (int kbi = 0; kbi < 2; ++kbi) {
              const int kb = 2 * q + kbi;
              const uint4 w = wv[kb];
              uint32_t a0, a1;
              decode_tables((shw[kb >> 2] >> (2 * (kb & 3))) & 3u, a0, a1);
              // columns 8*kbi + 0..3: k 0..15 of the block, 8*kbi + 4..7: k 16..31
              dec8(w.x, a0, a1, v[8 * kbi + 0], v[8 * kbi + 4]);
              dec8(w.y, a0, a1, v[8 * kbi + 1], v[8 * kbi + 5]);
              dec8(w.z, a0, a1, v[8 * kbi + 2], v[8 * kbi + 6]);
              dec8(w.w, a0, a1, v[8 * kbi + 3], v[8 * kbi + 7]);
            }
            tmem_st_x16(tcol + 16 * q, v);
          }
          // The packed slot goes back to the TMA producer only after the
          // decode has consumed the loaded registers.  Handing it back right
          // after issuing the shared-memory loads let a refill overwrite
          // bytes a lane had not read yet (one warp's 32 weight rows of a
          // stage decoded from the next stage's codes, seen as one corrupt
          // TMEM quarter per item in repeated full-size runs).
          __syncwarp();
          if (lane == 0) mbar_arrive(pk_empty(sp));
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) arrive_leader(a_full(sa));
          if (lane == 0 && quarter == 0) DSV4_TRACE_EV(5, gs);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(sh_empty(cc % SHS));
      }
      g += nks;
      s_first -= nks_mod;
      if (s_first < 0) s_first += G;
    }
  }
  tc_fence_before();
  __syncthreads();
  // CTA pairs: neither CTA leaves while the other may still arrive on its
  // barriers or read its shared memory
  if constexpr (kPair) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (kPair)
      tmem_dealloc_pair(tmem, C::kTmemCols);
    else
      tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace dsv4
