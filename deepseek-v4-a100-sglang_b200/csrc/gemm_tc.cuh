// MXFP4-weight x INT8-activation GEMM on the 5th-generation tensor core.
//
// One kernel serves the dense GEMM (reference DENSE_ENTRY:334-433), the
// grouped MoE GEMMs W13 / W2 (reference MOE_ENTRY:146-272, MOE_CORE:380-646)
// and the W13 GEMM with a fused SwiGLU epilogue (reference PYMOE:916-935).
//
// Orientation ("swap-AB"): the decoded weight tile is the MMA A operand
// (M = 128 weight rows = output channels), the gathered token rows are the
// B operand (N = 16..256 tokens), K-major both, int32 accumulators in TMEM
// laid out [channel lane][token column].  One weight tile, once decoded,
// serves every token of the tile.
//
// Warp roles (block = (4 + DECODE_WARPS) warps):
//   warp 0         bulk-copy producer: packed FP4 codes + 2-bit shifts of the
//                  weight tile, 128 K per stage, into the packed ring
//   warp 1         TMEM allocator and single-thread tcgen05.mma issuer
//   warps 2..3     activation gather (cp.async, 16 B, zero-fill) into the
//                  SW128 K-major B ring
//   warps 4..      FP4 -> INT8 decode from the packed ring into the SW128
//                  K-major A ring; afterwards the epilogue (TMEM -> regs ->
//                  scales -> bf16 / int32 / SwiGLU -> global)
#pragma once

#include "common.cuh"

namespace dsv4 {

enum Epilogue : int { kEpiBf16 = 0, kEpiI32 = 1, kEpiSwiglu = 2 };

struct TcGemmParams {
  // activations
  const int8_t* a;
  const float* a_scale;
  int64_t lda;
  int64_t a_rows;
  // weights in the repacked layout
  const uint8_t* b_packed;  // [E][KB][NG8][128]
  const uint8_t* b_shift;   // [E][SS][NG8][8]
  const float* cs;          // [E][N]
  int64_t b_expert_stride;  // bytes per expert in b_packed
  int64_t s_expert_stride;  // bytes per expert in b_shift
  int n;                    // weight rows (output channels) per expert
  int ng8;                  // ceil(n / 8)
  int inter;                // SwiGLU: intermediate size (gate rows [0,I), up rows [I,2I))
  int k_stages;             // K / 128
  int stages_per_split;
  // token rows of each tile
  int moe;                  // 0: dense rows, 1: rows from the aligned permutation
  int m;                    // dense: number of rows
  const int32_t* sorted_ids;
  const int32_t* expert_ids;
  const int32_t* ntpp;      // num_tokens_post_padded[0]
  int block_m;
  int topk;
  int num_valid;
  int src_is_slot;
  // outputs
  __nv_bfloat16* out;
  int64_t ldo;
  int32_t* out_i32;
  int64_t split_stride;
  float clamp_limit;
  int has_clamp;
};

template <int TN>
struct TcGemmCfg {
  static constexpr int kStagesAB = 3;
  static constexpr int kStagesP = 4;
  static constexpr int kABytes = 128 * 128;     // 128 weight rows x 128 K (int8)
  static constexpr int kBBytes = TN * 128;      // TN token rows x 128 K (int8)
  static constexpr int kPBytes = 128 * 128 / 2; // packed FP4 codes of one stage
  static constexpr int kShBytes = 128;
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kStagesAB * kABytes;
  static constexpr int kOffP = kOffB + kStagesAB * kBBytes;
  static constexpr int kOffSh = kOffP + kStagesP * kPBytes;
  static constexpr int kOffBar = kOffSh + kStagesP * kShBytes;
  static constexpr int kNumBars = 2 * kStagesP + 2 * kStagesAB + 1;
  static constexpr int kOffMeta = kOffBar + kNumBars * 8;
  static constexpr int kOffSrc = kOffMeta;
  static constexpr int kOffOrow = kOffSrc + TN * 4;
  static constexpr int kOffAsc = kOffOrow + TN * 4;
  static constexpr int kOffMisc = kOffAsc + TN * 4;  // tmem addr, last valid column
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kSmemLaunch = kBytes + 1024;  // slack for 1024-B alignment
  static constexpr int kTmemCols = TN < 32 ? 32 : TN;
  static_assert(TN % 16 == 0 && TN >= 16 && TN <= 256, "token tile");
  static_assert(kStagesAB * kABytes % 1024 == 0 && kBBytes % 1024 == 0, "alignment");
};

__device__ __forceinline__ __nv_bfloat16 f2bf(float v) { return __float2bfloat16_rn(v); }

template <int TN, int EPI, int DW>
__global__ void __launch_bounds__((4 + DW) * 32, DW == 4 ? 2 : 1)
mxfp4_int8_tc_gemm_kernel(const TcGemmParams p) {
  using C = TcGemmCfg<TN>;
  constexpr int S = C::kStagesAB;
  constexpr int SP = C::kStagesP;
  constexpr int kThreads = (4 + DW) * 32;
  static_assert(DW == 4 || DW == 8, "decode warps");

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  // ---- tile coordinates (uniform exits before any barrier / TMEM use) ----
  const int tile_x = blockIdx.x;
  const int tile_y = blockIdx.y;
  int expert = 0;
  if (p.moe) {
    if (tile_x * p.block_m >= __ldg(p.ntpp)) return;
    expert = __ldg(p.expert_ids + tile_x);
    if (expert < 0) return;
  }
  const int ks_begin = blockIdx.z * p.stages_per_split;
  const int ks_end = min(p.k_stages, ks_begin + p.stages_per_split);
  const int nks = ks_end - ks_begin;
  if (nks <= 0) return;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  const uint32_t bar0 = smem_u32(bars);
  auto pk_full = [&](int s) { return bar0 + 8u * s; };
  auto pk_empty = [&](int s) { return bar0 + 8u * (SP + s); };
  auto ab_full = [&](int s) { return bar0 + 8u * (2 * SP + s); };
  auto ab_empty = [&](int s) { return bar0 + 8u * (2 * SP + S + s); };
  const uint32_t acc_full = bar0 + 8u * (2 * SP + 2 * S);
  int* s_src = reinterpret_cast<int*>(smem + C::kOffSrc);
  int* s_orow = reinterpret_cast<int*>(smem + C::kOffOrow);
  float* s_asc = reinterpret_cast<float*>(smem + C::kOffAsc);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  int* s_last = reinterpret_cast<int*>(smem + C::kOffMisc + 4);

  if (tid == 0) {
    for (int s = 0; s < SP; ++s) {
      mbar_init(pk_full(s), 1);
      mbar_init(pk_empty(s), DW);
    }
    for (int s = 0; s < S; ++s) {
      mbar_init(ab_full(s), DW + 2);
      mbar_init(ab_empty(s), 1);
    }
    mbar_init(acc_full, 1);
    *s_last = -1;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(s_tmem), C::kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();

  // ---- token rows of this tile ----
  for (int j = tid; j < TN; j += kThreads) {
    int src = -1, orow = -1;
    float asc = 0.f;
    if (p.moe) {
      const int pos = tile_x * p.block_m + j;
      if (j < p.block_m) {
        const int slot = __ldg(p.sorted_ids + pos);
        if (slot >= 0 && slot < p.num_valid) {
          src = p.src_is_slot ? slot : slot / p.topk;
          orow = slot;
        }
      }
    } else {
      const int m = tile_x * TN + j;
      if (m < p.m) {
        src = m;
        orow = m;
      }
    }
    if (src >= p.a_rows) src = -1, orow = -1;
    if (src >= 0) {
      asc = p.a_scale != nullptr ? __ldg(p.a_scale + src) : 0.f;
      atomicMax(s_last, j);
    }
    s_src[j] = src;
    s_orow[j] = orow;
    s_asc[j] = asc;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const int last = *s_last;
  const int n_mma = ((last + 16) / 16) * 16;  // columns the MMA computes (>= 16)

  if (last >= 0) {
    // weight row groups of this tile
    int g0, g1;
    if (EPI == kEpiSwiglu) {
      g0 = (tile_y * 64) >> 3;             // gate rows j0 .. j0+63
      g1 = (p.inter + tile_y * 64) >> 3;   // up rows I+j0 .. I+j0+63
    } else {
      g0 = tile_y * 16;                    // rows 128*tile_y ..
      g1 = g0 + 8;
    }
    const uint8_t* bp = p.b_packed + static_cast<int64_t>(expert) * p.b_expert_stride;
    const uint8_t* bs = p.b_shift + static_cast<int64_t>(expert) * p.s_expert_stride;

    if (warp == 0) {
      // ------------------------- bulk-copy producer -------------------------
      if (lane == 0) {
        const uint64_t pol = l2_policy_evict_first();
        for (int it = 0; it < nks; ++it) {
          const int sp = it % SP;
          const uint32_t ph = (it / SP) & 1;
          mbar_wait(pk_empty(sp), ph ^ 1, kErrWaitPackedEmpty);
          mbar_arrive_expect_tx(pk_full(sp), C::kPBytes + C::kShBytes);
          const int ks = ks_begin + it;
          const uint32_t dstp = smem_u32(smem + C::kOffP + sp * C::kPBytes);
          for (int kb = 0; kb < 4; ++kb) {
            const int64_t kbg = static_cast<int64_t>(ks) * 4 + kb;
            const uint8_t* src0 = bp + (kbg * p.ng8 + g0) * 128;
            const uint8_t* src1 = bp + (kbg * p.ng8 + g1) * 128;
            bulk_g2s(dstp + kb * 2048, src0, 1024, pk_full(sp), pol);
            bulk_g2s(dstp + kb * 2048 + 1024, src1, 1024, pk_full(sp), pol);
          }
          const uint32_t dsts = smem_u32(smem + C::kOffSh + sp * C::kShBytes);
          bulk_g2s(dsts, bs + (static_cast<int64_t>(ks) * p.ng8 + g0) * 8, 64, pk_full(sp), pol);
          bulk_g2s(dsts + 64, bs + (static_cast<int64_t>(ks) * p.ng8 + g1) * 8, 64, pk_full(sp),
                   pol);
        }
      }
    } else if (warp == 1) {
      // ----------------------------- MMA issuer -----------------------------
      if (lane == 0) {
        const uint32_t idesc = idesc_i8(128, n_mma);
        for (int it = 0; it < nks; ++it) {
          const int sa = it % S;
          const uint32_t ph = (it / S) & 1;
          mbar_wait(ab_full(sa), ph, kErrWaitAbFull);
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + C::kOffA + sa * C::kABytes);
          const uint32_t b_base = smem_u32(smem + C::kOffB + sa * C::kBBytes);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            mma_i8(tmem, smem_desc_sw128(a_base + kk * 32), smem_desc_sw128(b_base + kk * 32),
                   idesc, (it > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(ab_empty(sa));
        }
        mma_commit(acc_full);
      }
    } else if (warp < 4) {
      // -------------------------- activation gather -------------------------
      const int gt = tid - 64;
      constexpr int LAG = 1;
      for (int it = 0; it < nks; ++it) {
        const int sa = it % S;
        const uint32_t ph = (it / S) & 1;
        mbar_wait(ab_empty(sa), ph ^ 1, kErrWaitAbEmpty);
        const int64_t k0 = static_cast<int64_t>(ks_begin + it) * 128;
        const uint32_t b_base = smem_u32(smem + C::kOffB + sa * C::kBBytes);
        for (int idx = gt; idx < n_mma * 8; idx += 64) {
          const int j = idx >> 3;
          const int c = idx & 7;
          const int src = s_src[j];
          const uint32_t dst = b_base + (j >> 3) * 1024 + (j & 7) * 128 + ((c ^ (j & 7)) << 4);
          const int8_t* g = src >= 0 ? p.a + static_cast<int64_t>(src) * p.lda + k0 + c * 16 : p.a;
          cp_async_16(dst, g, src >= 0 ? 16u : 0u);
        }
        cp_async_commit();
        if (it >= LAG) {
          cp_async_wait<LAG>();
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(ab_full((it - LAG) % S));
        }
      }
      cp_async_wait<0>();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        for (int it = (nks > LAG ? nks - LAG : 0); it < nks; ++it) mbar_arrive(ab_full(it % S));
      }
    } else {
      // ------------------------ FP4 -> INT8 decode -------------------------
      const int d = tid - 128;
      const int row = d & 127;
      constexpr int kKbPerThread = 16 / DW;  // 4 (DW=4) or 2 (DW=8)
      const int kb_begin = (DW == 8) ? (d >> 7) * 2 : 0;
      const int rsw = row & 7;
      for (int it = 0; it < nks; ++it) {
        const int sp = it % SP;
        const int sa = it % S;
        mbar_wait(pk_full(sp), (it / SP) & 1, kErrWaitPackedFull);
        mbar_wait(ab_empty(sa), ((it / S) & 1) ^ 1, kErrWaitAbEmpty);
        const uint8_t* P = smem + C::kOffP + sp * C::kPBytes;
        const uint32_t shb = smem[C::kOffSh + sp * C::kShBytes + row];
        uint8_t* A = smem + C::kOffA + sa * C::kABytes + (row >> 3) * 1024 + rsw * 128;
#pragma unroll
        for (int kbi = 0; kbi < kKbPerThread; ++kbi) {
          const int kb = kb_begin + kbi;
          const uint4 w = *reinterpret_cast<const uint4*>(P + (kb * 128 + row) * 16);
          uint32_t t0, t1;
          decode_tables((shb >> (2 * kb)) & 3u, t0, t1);
          uint4 lo, hi;
          decode8(w.x, t0, t1, lo.x, hi.x);
          decode8(w.y, t0, t1, lo.y, hi.y);
          decode8(w.z, t0, t1, lo.z, hi.z);
          decode8(w.w, t0, t1, lo.w, hi.w);
          *reinterpret_cast<uint4*>(A + (((2 * kb) ^ rsw) << 4)) = lo;
          *reinterpret_cast<uint4*>(A + (((2 * kb + 1) ^ rsw) << 4)) = hi;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(pk_empty(sp));
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(ab_full(sa));
      }

      // ------------------------------ epilogue ------------------------------
      mbar_wait(acc_full, 0, kErrWaitAccFull);
      tc_fence_after();
      const int quarter = warp & 3;          // TMEM lanes 32*quarter .. +31
      const int grp = (warp - 4) >> 2;       // epilogue group (column interleave)
      constexpr int kGroups = DW / 4;
      const int row_local = quarter * 32 + lane;
      const uint32_t t_row = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
      const float* cs_e = p.cs + static_cast<int64_t>(expert) * p.n;

      if (EPI == kEpiSwiglu) {
        const bool is_up = row_local >= 64;
        const int i_local = row_local & 63;
        const int j0 = tile_y * 64;
        const float csn = __ldg(cs_e + (is_up ? p.inter : 0) + j0 + i_local);
        // staging: 16 columns x 128 rows bf16, one buffer per epilogue group,
        // in the (now idle) A ring.
        __nv_bfloat16* stg =
            reinterpret_cast<__nv_bfloat16*>(smem + C::kOffA) + grp * (16 * 128);
        const int e = tid - 128 - grp * 128;  // 0..127 inside the group
        const float lim = p.has_clamp ? __bfloat162float(f2bf(p.clamp_limit)) : 0.f;
        for (int c0 = grp * 16; c0 < n_mma; c0 += 16 * kGroups) {
          int32_t v[16];
          tmem_ld_x16(t_row + c0, v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float x = __fmul_rn(__fmul_rn(__int2float_rn(v[j]), s_asc[c0 + j]), csn);
            stg[j * 128 + row_local] = f2bf(x);
          }
          named_bar_sync(1 + grp, 128);
          const int col = c0 + (e >> 3);
          const int i0 = (e & 7) * 8;
          const int orow = s_orow[col];
          if (orow >= 0) {
            __align__(16) __nv_bfloat16 h[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              float g = __bfloat162float(stg[(e >> 3) * 128 + i0 + u]);
              float up = __bfloat162float(stg[(e >> 3) * 128 + 64 + i0 + u]);
              if (p.has_clamp) {
                g = fminf(g, lim);
                up = fminf(fmaxf(up, -lim), lim);
              }
              const float sg = __bfloat162float(f2bf(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g)))));
              h[u] = f2bf(__fmul_rn(sg, up));
            }
            *reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(orow) * p.ldo + j0 + i0) =
                *reinterpret_cast<const uint4*>(h);
          }
          named_bar_sync(1 + grp, 128);
        }
      } else {
        const int n_g = tile_y * 128 + row_local;
        const float csn = (EPI == kEpiBf16) ? __ldg(cs_e + n_g) : 0.f;
        for (int c0 = grp * 16; c0 < n_mma; c0 += 16 * kGroups) {
          int32_t v[16];
          tmem_ld_x16(t_row + c0, v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int orow = s_orow[c0 + j];
            if (orow < 0) continue;
            if (EPI == kEpiBf16) {
              const float x = __fmul_rn(__fmul_rn(__int2float_rn(v[j]), s_asc[c0 + j]), csn);
              p.out[static_cast<int64_t>(orow) * p.ldo + n_g] = f2bf(x);
            } else {
              p.out_i32[static_cast<int64_t>(blockIdx.z) * p.split_stride +
                        static_cast<int64_t>(orow) * p.ldo + n_g] = v[j];
            }
          }
        }
      }
      tc_fence_before();
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace dsv4
