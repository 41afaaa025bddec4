// Memory-bound kernels of the MoE path: per-token INT8 quantisation, expert
// align (histogram / padded prefix sum / stable permutation), the load-time
// MXFP4 -> INT8-decodable repack, the top-k combine and the dense split-K
// reduce.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace dsv4 {

// ---------------------------------------------------------------------------
// a1. per-token INT8 quantisation (reference PYMOE:53-126).
// One warp per row.  scale = max|x| / 127 (IEEE division; 0 -> 1.0),
// q = clamp(rne(x / scale), -127, 127).
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

__device__ __forceinline__ float clampf_abs(float x, float c) {
  return c > 0.f ? fminf(fmaxf(x, -c), c) : x;
}

__device__ __forceinline__ int8_t quant1(float x, float s) {
  int q = __float2int_rn(__fdiv_rn(x, s));
  q = max(-127, min(127, q));
  return static_cast<int8_t>(q);
}

template <typename T>
__global__ void __launch_bounds__(256) quant_rows_kernel(const T* __restrict__ a, int64_t m,
                                                         int64_t k, int64_t lda, float clamp_abs,
                                                         int8_t* __restrict__ q,
                                                         float* __restrict__ scale) {
  pdl_entry();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= m) return;
  const T* x = a + row * lda;
  int8_t* qr = q + row * k;
  const bool vec = (sizeof(T) == 2) && (k % 8 == 0) && (lda % 8 == 0) &&
                   ((reinterpret_cast<uintptr_t>(a) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(q) & 7) == 0);
  float amax = 0.f;
  if (vec) {
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    for (int64_t i = lane; i < k / 8; i += 32) {
      uint4 u = __ldg(xv + i);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(clampf_abs(to_f32<T>(e[j]), clamp_abs)));
    }
  } else {
    for (int64_t i = lane; i < k; i += 32) amax = fmaxf(amax, fabsf(clampf_abs(to_f32<T>(x[i]), clamp_abs)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  float s = __fdiv_rn(amax, 127.0f);
  if (s == 0.0f) s = 1.0f;
  if (vec) {
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    for (int64_t i = lane; i < k / 8; i += 32) {
      uint4 u = __ldg(xv + i);
      const T* e = reinterpret_cast<const T*>(&u);
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        lo |= (static_cast<uint32_t>(static_cast<uint8_t>(quant1(clampf_abs(to_f32<T>(e[j]), clamp_abs), s)))) << (8 * j);
        hi |= (static_cast<uint32_t>(static_cast<uint8_t>(quant1(clampf_abs(to_f32<T>(e[j + 4]), clamp_abs), s)))) << (8 * j);
      }
      reinterpret_cast<uint2*>(qr)[i] = make_uint2(lo, hi);
    }
  } else {
    for (int64_t i = lane; i < k; i += 32) qr[i] = quant1(clampf_abs(to_f32<T>(x[i]), clamp_abs), s);
  }
  if (lane == 0) scale[row] = s;
}

// Register-resident variant for bf16/fp16 rows with K % 8 == 0: each row is
// read once (uint4 per 8 elements) by RT threads (RT = 32 or 128), reduced,
// then quantised from registers.  Same arithmetic as quant_rows_kernel.
// With `sorted` set the rows are expert-sorted positions: only positions below
// num_tokens_post_padded holding a routed slot (< num_valid) are quantised, q
// is written K-chunk-major, [K/128][cm_rows][128], the layout the GEMM's
// sorted-row mode loads with one copy per stage, and rowsum[row] receives the
// sum of the row's int8 values (for the GEMM's biased-unsigned decode).
// Warp-per-row instances (K <= 2048: the sorted requant) are held to six
// CTAs per SM: more resident warps outweigh the few spilled registers
// (requant at M=8192 187 -> 172 us); the 128-thread rows keep the default.
template <typename T, int RT, int VPT>
__global__ void __launch_bounds__(256, RT == 32 ? 6 : 0) quant_rows_reg_kernel(const T* __restrict__ a, int64_t m,
                                                             int64_t k, int64_t lda,
                                                             float clamp_abs,
                                                             int8_t* __restrict__ q,
                                                             float* __restrict__ scale,
                                                             const int32_t* __restrict__ sorted = nullptr,
                                                             const int32_t* __restrict__ ntpp = nullptr,
                                                             int num_valid = 0, int64_t cm_rows = 0,
                                                             int32_t* __restrict__ rowsum = nullptr,
                                                             int gather_topk = 0) {
  pdl_entry();
  constexpr int kRowsPerCta = 256 / RT;
  __shared__ float red[256 / 32];
  __shared__ int red_i[256 / 32];
  const int r_local = threadIdx.x / RT;
  const int lt = threadIdx.x % RT;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowsPerCta + r_local;
  bool active = row < m;
  // source row: the row itself, or (gather_topk > 0, the fused quantise +
  // sort of the token rows) the token of the routed slot at this position
  int64_t src_row = row;
  if (sorted != nullptr && active) {
    const int slot = row < __ldg(ntpp) ? __ldg(sorted + row) : -1;
    active = slot >= 0 && slot < num_valid;
    if (gather_topk > 0) src_row = active ? slot / gather_topk : 0;
  }
  const int nv = static_cast<int>(k / 8);
  uint4 u[VPT];
  float amax = 0.f;
  if (active) {
    const uint4* xv = reinterpret_cast<const uint4*>(a + src_row * lda);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = lt + i * RT;
      if (idx < nv) {
        u[i] = __ldg(xv + idx);
        const T* e = reinterpret_cast<const T*>(&u[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(clampf_abs(to_f32<T>(e[j]), clamp_abs)));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (RT > 32) {
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    const int w0 = (r_local * RT) >> 5;
    amax = 0.f;
#pragma unroll
    for (int w = 0; w < RT / 32; ++w) amax = fmaxf(amax, red[w0 + w]);
  }
  if (!active && rowsum == nullptr) return;
  float sc = __fdiv_rn(amax, 127.0f);
  if (sc == 0.0f) sc = 1.0f;
  uint2* qr = reinterpret_cast<uint2*>(q + row * k);
  int qsum = 0;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = lt + i * RT;
    if (active && idx < nv) {
      // 8 elements at k = 8 idx; K-chunk-major: chunk idx / 16, byte 8 (idx % 16)
      uint2* dst = cm_rows == 0
                       ? qr + idx
                       : reinterpret_cast<uint2*>(q + (idx >> 4) * cm_rows * 128 + row * 128 + (idx & 15) * 8);
      const T* e = reinterpret_cast<const T*>(&u[i]);
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        lo |= static_cast<uint32_t>(static_cast<uint8_t>(quant1(clampf_abs(to_f32<T>(e[j]), clamp_abs), sc))) << (8 * j);
        hi |= static_cast<uint32_t>(static_cast<uint8_t>(quant1(clampf_abs(to_f32<T>(e[j + 4]), clamp_abs), sc))) << (8 * j);
      }
      *dst = make_uint2(lo, hi);
      qsum = __dp4a(static_cast<int>(lo), 0x01010101, qsum);
      qsum = __dp4a(static_cast<int>(hi), 0x01010101, qsum);
    }
  }
  if (rowsum != nullptr) {  // every thread of the CTA reaches this point
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, o);
    if (RT > 32) {
      if ((threadIdx.x & 31) == 0) red_i[threadIdx.x >> 5] = qsum;
      __syncthreads();
      const int w0 = (r_local * RT) >> 5;
      qsum = 0;
#pragma unroll
      for (int w = 0; w < RT / 32; ++w) qsum += red_i[w0 + w];
    }
    if (active && lt == 0) rowsum[row] = qsum;
  }
  if (active && lt == 0) scale[row] = sc;
}

// Expert-sorted copy of quantised rows: position pos < num_tokens_post_padded
// holding routed slot s (< num_valid) receives row (s / topk, or s when the
// rows are slots) of a_q and its scale, K-chunk-major [K/128][cap][128].
// Padding positions are left unwritten (their MMA columns are never stored).
// Source rows are lda bytes apart and their scales scale_stride floats apart
// (rows received packed with their metadata).  With sorted == nullptr the
// permutation is the identity over cap positions (dense activations into the
// K-chunk-major layout; out_scale may then be null).  One warp per position,
// 16 B per lane.
__global__ void __launch_bounds__(256) sort_rows_kernel(const int8_t* __restrict__ a,
                                                        const float* __restrict__ a_scale,
                                                        int64_t a_rows, int64_t k,
                                                        int64_t lda, int64_t scale_stride,
                                                        const int32_t* __restrict__ sorted,
                                                        const int32_t* __restrict__ ntpp,
                                                        int64_t cap, int topk, int src_is_slot,
                                                        int num_valid, int8_t* __restrict__ out,
                                                        float* __restrict__ out_scale,
                                                        int32_t* __restrict__ out_rowsum) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const int64_t n = ntpp != nullptr ? min(cap, static_cast<int64_t>(__ldg(ntpp))) : cap;
  const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int nv = static_cast<int>(k / 16);
  for (int64_t pos = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; pos < n;
       pos += nw) {
    // no permutation (sorted == nullptr): position p holds row p
    const int slot = sorted != nullptr ? __ldg(sorted + pos) : static_cast<int>(pos);
    if (slot < 0 || slot >= num_valid) continue;
    const int64_t src = sorted == nullptr || src_is_slot ? slot : slot / topk;
    if (src >= a_rows) continue;
    const int4* row = reinterpret_cast<const int4*>(a + src * lda);
    int sum = 0;
    // four 16-byte loads in flight per lane
    int c = lane;
    for (; c + 96 < nv; c += 128) {
      int4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldg(row + c + 32 * u);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int cc = c + 32 * u;
        *reinterpret_cast<int4*>(out + (cc >> 3) * cap * 128 + pos * 128 + (cc & 7) * 16) = v[u];
        sum = __dp4a(v[u].x, 0x01010101, __dp4a(v[u].y, 0x01010101, __dp4a(v[u].z, 0x01010101, __dp4a(v[u].w, 0x01010101, sum))));
      }
    }
    for (; c < nv; c += 32) {
      const int4 v = __ldg(row + c);
      *reinterpret_cast<int4*>(out + (c >> 3) * cap * 128 + pos * 128 + (c & 7) * 16) = v;
      sum = __dp4a(v.x, 0x01010101, __dp4a(v.y, 0x01010101, __dp4a(v.z, 0x01010101, __dp4a(v.w, 0x01010101, sum))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      if (out_scale != nullptr) out_scale[pos] = __ldg(a_scale + src * scale_stride);
      out_rowsum[pos] = sum;
    }
  }
}

// Quantise + scatter into expert order: the inverse of the fused quantise +
// sort.  Each token row is read and quantised once (the arithmetic of
// quant_rows_kernel), and its int8 values, scale and int8 row sum are written
// to the sorted position of each of its topk routed slots, K-chunk-major
// [K/128][cap][128]: slot_pos[t * topk + j] (-1: not placed).  Slots at or
// past num_valid are skipped.  The outputs equal quantise-then-sort_rows bit
// for bit; padding positions are left unwritten.  RT threads per row,
// 256 / RT rows per CTA, VPT 16-byte loads per thread (K <= 8 RT VPT).
template <typename T, int RT, int VPT>
__global__ void __launch_bounds__(256) quant_scatter_kernel(const T* __restrict__ a, int64_t m,
                                                            int64_t k, int64_t lda,
                                                            const int32_t* __restrict__ slot_pos,
                                                            int topk, int num_valid, int64_t cap,
                                                            int8_t* __restrict__ q,
                                                            float* __restrict__ scale,
                                                            int32_t* __restrict__ rowsum) {
  pdl_entry();
  constexpr int kRowsPerCta = 256 / RT;
  __shared__ float red[256 / 32];
  __shared__ int red_i[256 / 32];
  const int r_local = threadIdx.x / RT;
  const int lt = threadIdx.x % RT;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowsPerCta + r_local;
  const bool active = row < m;
  const int nv = static_cast<int>(k / 8);
  uint4 u[VPT];
  float amax = 0.f;
  if (active) {
    const uint4* xv = reinterpret_cast<const uint4*>(a + row * lda);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = lt + i * RT;
      if (idx < nv) {
        u[i] = __ldg(xv + idx);
        const T* e = reinterpret_cast<const T*>(&u[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(to_f32<T>(e[j])));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (RT > 32) {
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    const int w0 = (r_local * RT) >> 5;
    amax = 0.f;
#pragma unroll
    for (int w = 0; w < RT / 32; ++w) amax = fmaxf(amax, red[w0 + w]);
  }
  float sc = __fdiv_rn(amax, 127.0f);
  if (sc == 0.0f) sc = 1.0f;
  uint2 packed[VPT];
  int qsum = 0;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = lt + i * RT;
    packed[i] = make_uint2(0u, 0u);
    if (active && idx < nv) {
      const T* e = reinterpret_cast<const T*>(&u[i]);
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        lo |= static_cast<uint32_t>(static_cast<uint8_t>(quant1(to_f32<T>(e[j]), sc))) << (8 * j);
        hi |= static_cast<uint32_t>(static_cast<uint8_t>(quant1(to_f32<T>(e[j + 4]), sc))) << (8 * j);
      }
      packed[i] = make_uint2(lo, hi);
      qsum = __dp4a(static_cast<int>(lo), 0x01010101, qsum);
      qsum = __dp4a(static_cast<int>(hi), 0x01010101, qsum);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, o);
  if (RT > 32) {
    if ((threadIdx.x & 31) == 0) red_i[threadIdx.x >> 5] = qsum;
    __syncthreads();
    const int w0 = (r_local * RT) >> 5;
    qsum = 0;
#pragma unroll
    for (int w = 0; w < RT / 32; ++w) qsum += red_i[w0 + w];
  }
  if (!active) return;
  for (int j = 0; j < topk; ++j) {
    const int64_t slot = row * topk + j;
    if (slot >= num_valid) break;
    const int pos = __ldg(slot_pos + slot);
    if (pos < 0 || pos >= cap) continue;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = lt + i * RT;
      if (idx < nv)
        *reinterpret_cast<uint2*>(q + (idx >> 4) * cap * 128 + static_cast<int64_t>(pos) * 128 +
                                  (idx & 15) * 8) = packed[i];
    }
    if (lt == 0) {
      scale[pos] = sc;
      rowsum[pos] = qsum;
    }
  }
}

// ---------------------------------------------------------------------------
// Router top-k (the DeepSeek routing SGLang computes before the MoE call,
// reference PATCH:505-507): score = sigmoid(logit); the top-k experts by
// score + bias (bias used for selection only); weight = chosen score,
// renormalised to sum 1 when asked, times `scale`.  One warp per token, EPL
// experts per lane in registers; k rounds of a warp argmax (ties: lower
// expert index), so the k results come out in descending order.
// One token's routing by one warp; lanes r < topk end with (my_id, my_w) of
// the r-th choice.
template <typename T, int EPL>
__device__ __forceinline__ void router_row(const T* __restrict__ logits, int64_t row, int e,
                                           const float* __restrict__ bias, int topk,
                                           int renormalize, float scale, int lane, int& out_id,
                                           float& out_w) {
  float sel[EPL], sc[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int x = j * 32 + lane;
    if (x < e) {
      const float l = to_f32<T>(logits[row * e + x]);
      sc[j] = 1.0f / (1.0f + expf(-l));
      sel[j] = sc[j] + (bias != nullptr ? bias[x] : 0.f);
    } else {
      sc[j] = 0.f;
      sel[j] = -INFINITY;
    }
  }
  float wsum = 0.f, my_w = 0.f;
  int my_id = -1;
  for (int r = 0; r < topk; ++r) {
    float bv = -INFINITY;
    int bx = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int x = j * 32 + lane;
      if (sel[j] > bv || (sel[j] == bv && x < bx)) bv = sel[j], bx = x;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int ox = __shfl_xor_sync(0xffffffffu, bx, o);
      if (ov > bv || (ov == bv && ox < bx)) bv = ov, bx = ox;
    }
    // the owning lane clears the winner and broadcasts its score
    float w = 0.f;
    if ((bx & 31) == lane) {
#pragma unroll
      for (int j = 0; j < EPL; ++j)
        if (j == (bx >> 5)) w = sc[j], sel[j] = -INFINITY;
    }
    w = __shfl_sync(0xffffffffu, w, bx & 31);
    wsum += w;
    if (lane == r) my_w = w, my_id = bx;
  }
  out_id = my_id;
  out_w = (renormalize ? my_w / wsum : my_w) * scale;
}

template <typename T, int EPL>
__global__ void __launch_bounds__(256) router_topk_kernel(const T* __restrict__ logits, int64_t m,
                                                          int e, const float* __restrict__ bias,
                                                          int topk, int renormalize, float scale,
                                                          int32_t* __restrict__ ids,
                                                          float* __restrict__ weights) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= m) return;
  int id;
  float w;
  router_row<T, EPL>(logits, row, e, bias, topk, renormalize, scale, lane, id, w);
  if (lane < topk) {
    ids[row * topk + lane] = id;
    weights[row * topk + lane] = w;
  }
}

// ---------------------------------------------------------------------------
// a5. expert align (reference call site PYMOE:842-869, library
// sgl_kernel.moe_align_block_size).  One CTA of 1024 threads:
//   1. each warp owns a contiguous segment of the flattened ids and counts
//      its experts (shared atomics; counts are order-free),
//   2. per expert: exclusive prefix over warps (stable placement bases),
//   3. block-padded exclusive prefix over experts,
//   4. each warp walks its segment in id order, 32 at a time; __match_any
//      groups equal experts, the rank among lower lanes gives the position.
// Result: inside an expert segment slot ids increase (stable order); padding
// value is numel; ids outside [0, E) are dropped; expert_ids of blocks past
// the padded total are -1.  Optionally slot_pos[i] = the position of slot i
// (-1 for a dropped id): the inverse permutation, for the quantise-scatter.
// ---------------------------------------------------------------------------
constexpr int kAlignThreads = 1024;

__global__ void __launch_bounds__(kAlignThreads, 1)
moe_align_kernel(const int32_t* __restrict__ ids, int numel, int num_experts, int block_m,
                 int32_t* __restrict__ sorted_ids, int sorted_cap, int32_t* __restrict__ expert_ids,
                 int expert_cap, int32_t* __restrict__ ntpp, int32_t* __restrict__ cumsum_out,
                 int32_t* __restrict__ slot_pos) {
  pdl_entry();
  extern __shared__ int sm_align[];
  const int E = num_experts;
  int* wc = sm_align;             // [32][E] per-warp counts, then placement cursors
  int* base = wc + 32 * E;        // [E + 1] padded exclusive prefix
  int* wsum = base + E + 1;       // [32] scan scratch
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int seg = (numel + 31) / 32;
  const int s_begin = min(numel, warp * seg);
  const int s_end = min(numel, s_begin + seg);

  for (int i = tid; i < 32 * E; i += kAlignThreads) wc[i] = 0;
  __syncthreads();
  for (int i = s_begin + lane; i < s_end; i += 32) {
    const int e = __ldg(ids + i);
    if (e >= 0 && e < E) atomicAdd(&wc[warp * E + e], 1);
  }
  __syncthreads();
  // per-expert prefix over warps; expert total into base[e]
  for (int e = tid; e < E; e += kAlignThreads) {
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = wc[w * E + e];
      wc[w * E + e] = run;
      run += c;
    }
    base[e] = run;
  }
  __syncthreads();
  // block-padded exclusive scan over experts (E <= 1024 -> one per thread)
  {
    const int cnt = tid < E ? base[tid] : 0;
    const int padded = (cnt + block_m - 1) / block_m * block_m;
    int v = padded;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += n;
    }
    if (lane == 31) wsum[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int w = wsum[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += n;
      }
      wsum[lane] = w;
    }
    __syncthreads();
    const int incl = v + (warp > 0 ? wsum[warp - 1] : 0);
    __syncthreads();
    if (tid < E) base[tid] = incl - padded;
    if (tid == E - 1) base[E] = incl;
    if (E == 0 && tid == 0) base[0] = 0;
  }
  __syncthreads();
  const int total = base[E];
  for (int i = tid; i < sorted_cap; i += kAlignThreads) sorted_ids[i] = numel;
  for (int b = tid; b < expert_cap; b += kAlignThreads) {
    int e = -1;
    const int pos = b * block_m;
    if (pos < total) {
      int lo = 0, hi = E - 1;  // last e with base[e] <= pos
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (base[mid] <= pos) lo = mid; else hi = mid - 1;
      }
      e = lo;
    }
    expert_ids[b] = e;
  }
  if (tid == 0) ntpp[0] = total;
  if (cumsum_out != nullptr)
    for (int e = tid; e <= E; e += kAlignThreads) cumsum_out[e] = base[e];
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int c = s_begin; c < s_end; c += 32) {
    const int i = c + lane;
    int e = i < s_end ? __ldg(ids + i) : -1;
    const bool valid = e >= 0 && e < E;
    const int key = valid ? e : (E + lane);  // unique key for invalid lanes
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int rank = __popc(peers & lt_mask);
    int pos = -1;
    if (valid) {
      pos = base[e] + wc[warp * E + e] + rank;
      if (pos < sorted_cap) sorted_ids[pos] = i; else pos = -1;
    }
    if (slot_pos != nullptr && i < s_end) slot_pos[i] = pos;
    __syncwarp();
    if (valid && rank == 0) wc[warp * E + e] += __popc(peers);
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// a3. MXFP4 -> INT8-decodable repack (reference PYMOE:378-572 Triton kernels,
// PYMOE:642-666 torch variant).  Load time only.
// ---------------------------------------------------------------------------
__global__ void repack_channel_shift_kernel(const uint8_t* __restrict__ scale, int64_t rows,
                                            int n, int kb_count, int ss, int ng8, int headroom,
                                            float* __restrict__ cs, uint8_t* __restrict__ shift2) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const uint8_t* sr = scale + row * kb_count;
  int mx = -32768;
  for (int kb = 0; kb < kb_count; ++kb) mx = max(mx, static_cast<int>(sr[kb]) - 127);
  cs[row] = ldexpf(0.5f, mx - headroom);
  const int64_t e = row / n;
  const int nn = static_cast<int>(row - e * n);
  const int g = nn >> 3, r = nn & 7;
  for (int sb = 0; sb < ss; ++sb) {
    uint32_t packed = 0;
    for (int i = 0; i < 4; ++i) {
      const int kb = sb * 4 + i;
      if (kb < kb_count) {
        const int delta = mx - (static_cast<int>(sr[kb]) - 127);
        const int sh = min(3, max(0, headroom - delta));
        packed |= static_cast<uint32_t>(sh) << (2 * i);
      }
    }
    shift2[((e * ss + sb) * ng8 + g) * 8 + r] = static_cast<uint8_t>(packed);
  }
}

__device__ __forceinline__ uint32_t remap_nibble(uint32_t nib, int exp, int max_exp, int headroom,
                                                 int half_even) {
  const uint32_t mag = nib & 7u;
  const uint32_t sign = nib & 8u;
  if (mag == 0) return 0u;
  const float q_abs = static_cast<float>((0x0C08060403020100ull >> (8 * mag)) & 0xFF);
  const int delta = max(max_exp - exp, 0);
  const int shift = min(3, max(0, headroom - delta));
  const float target = ldexpf(q_abs, headroom - delta);
  float ti = half_even ? fminf(rintf(target), 128.0f) : floorf(target + 0.5f);
  const float v = ldexpf(ti, -shift);
  uint32_t m = 7;
  if (v <= 10.0f) m = 6;
  if (v <= 7.0f) m = 5;
  if (v <= 5.0f) m = 4;
  if (v <= 3.5f) m = 3;
  if (v <= 2.5f) m = 2;
  if (v <= 1.5f) m = 1;
  if (v <= 0.5f) m = 0;
  return m | sign;
}

// One thread per 32-bit word of the packed layout: (e, kb, g, lane).
__global__ void repack_codes_kernel(const uint8_t* __restrict__ weight,
                                    const uint8_t* __restrict__ scale,
                                    const float* __restrict__ cs, int64_t total_words, int n,
                                    int kb_count, int ng8, int headroom, int half_even,
                                    uint32_t* __restrict__ out) {
  const int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (w >= total_words) return;
  const int lane = static_cast<int>(w & 31);
  const int64_t t1 = w >> 5;
  const int g = static_cast<int>(t1 % ng8);
  const int64_t t2 = t1 / ng8;
  const int kb = static_cast<int>(t2 % kb_count);
  const int64_t e = t2 / kb_count;
  const int nn = g * 8 + (lane >> 2);
  const int t = lane & 3;
  uint32_t word = 0;
  if (nn < n) {
    const int64_t row = e * n + nn;
    const int max_exp = ilogbf(cs[row]) + headroom + 1;
    const int exp = static_cast<int>(scale[row * kb_count + kb]) - 127;
    const uint8_t* src = weight + row * (kb_count * 16) + kb * 16;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int kk = (j < 2 ? 4 * t : 16 + 4 * t) + 2 * (j & 1);
      const uint32_t byte = src[kk >> 1];
      const uint32_t lo = remap_nibble(byte & 15u, exp, max_exp, headroom, half_even);
      const uint32_t hi = remap_nibble(byte >> 4, exp, max_exp, headroom, half_even);
      word |= (lo | (hi << 4)) << (8 * j);
    }
  }
  out[w] = word;
}

// ---------------------------------------------------------------------------
// a9. top-k combine (reference MOE_ENTRY:71-126) with the optional routed
// scaling of PYMOE:957-958 fused: out = bf16(bf16(sum_k fma) * rsf).
// One thread per (token, 8 columns).
// ---------------------------------------------------------------------------
__global__ void moe_reduce_kernel(const __nv_bfloat16* __restrict__ routed,
                                  const float* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                  int m_out, int n, int topk, int num_valid, float rsf,
                                  int apply_rsf) {
  pdl_entry();
  const int chunks = n / 8;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(m_out) * chunks) return;
  const int t = static_cast<int>(idx / chunks);
  const int c = static_cast<int>(idx - static_cast<int64_t>(t) * chunks);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int k = 0; k < topk; ++k) {
    const int slot = t * topk + k;
    if (slot >= num_valid) continue;
    const float wt = __ldg(w + slot);
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(routed + static_cast<int64_t>(slot) * n) + c);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = __fmaf_rn(__bfloat162float(e[i]), wt, acc[i]);
  }
  __align__(16) __nv_bfloat16 o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    __nv_bfloat16 b = __float2bfloat16_rn(acc[i]);
    if (apply_rsf) b = __float2bfloat16_rn(__fmul_rn(__bfloat162float(b), rsf));
    o[i] = b;
  }
  reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * n)[c] = *reinterpret_cast<uint4*>(o);
}

// Top-k combine that skips slots whose expert id is negative (expert held by
// another rank under expert parallelism; their routed rows are never
// written).  Otherwise identical to moe_reduce_kernel.
__global__ void moe_reduce_masked_kernel(const __nv_bfloat16* __restrict__ routed,
                                         const float* __restrict__ w,
                                         const int32_t* __restrict__ ids,
                                         __nv_bfloat16* __restrict__ out, int m_out, int n,
                                         int topk, int num_valid, float rsf, int apply_rsf) {
  pdl_entry();
  const int chunks = n / 8;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(m_out) * chunks) return;
  const int t = static_cast<int>(idx / chunks);
  const int c = static_cast<int>(idx - static_cast<int64_t>(t) * chunks);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int k = 0; k < topk; ++k) {
    const int slot = t * topk + k;
    if (slot >= num_valid || __ldg(ids + slot) < 0) continue;
    const float wt = __ldg(w + slot);
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(routed + static_cast<int64_t>(slot) * n) + c);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = __fmaf_rn(__bfloat162float(e[i]), wt, acc[i]);
  }
  __align__(16) __nv_bfloat16 o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    __nv_bfloat16 b = __float2bfloat16_rn(acc[i]);
    if (apply_rsf) b = __float2bfloat16_rn(__fmul_rn(__bfloat162float(b), rsf));
    o[i] = b;
  }
  reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * n)[c] = *reinterpret_cast<uint4*>(o);
}

// Row gather: dst row i (dst_stride bytes apart) = src[idx[i]] (row_bytes,
// a multiple of 16), or zeros where idx[i] < 0.
__global__ void gather_rows_kernel(const uint8_t* __restrict__ src, int64_t row_bytes,
                                   const int64_t* __restrict__ idx, int64_t n_rows,
                                   uint8_t* __restrict__ dst, int64_t dst_stride) {
  const int64_t vec = row_bytes / 16;
  const int64_t total = n_rows * vec;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / vec;
    const int64_t c = i - r * vec;
    const int64_t s = __ldg(idx + r);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (s >= 0) v = __ldg(reinterpret_cast<const uint4*>(src + s * row_bytes) + c);
    reinterpret_cast<uint4*>(dst + r * dst_stride)[c] = v;
  }
}

// Expert-parallel combine: out[t] = bf16(sum_r f32(partial[pos[t][r]])) over
// r = 0..world-1 in rank order (pos -1 = no partial from rank r), then the
// optional routed scaling in bf16.  One thread per (token, 8 columns).
__global__ void ep_combine_kernel(const __nv_bfloat16* __restrict__ partial,
                                  const int64_t* __restrict__ pos, int world,
                                  __nv_bfloat16* __restrict__ out, int m, int n, float rsf,
                                  int apply_rsf) {
  const int chunks = n / 8;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(m) * chunks) return;
  const int t = static_cast<int>(idx / chunks);
  const int c = static_cast<int>(idx - static_cast<int64_t>(t) * chunks);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int r = 0; r < world; ++r) {
    const int64_t p = __ldg(pos + static_cast<int64_t>(t) * world + r);
    if (p < 0) continue;
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(partial + p * n) + c);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __bfloat162float(e[i]));
  }
  __align__(16) __nv_bfloat16 o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    __nv_bfloat16 b = __float2bfloat16_rn(acc[i]);
    if (apply_rsf) b = __float2bfloat16_rn(__fmul_rn(__bfloat162float(b), rsf));
    o[i] = b;
  }
  reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * n)[c] = *reinterpret_cast<uint4*>(o);
}

// Expert-parallel plan for the fixed-capacity exchange (one CTA, any m <=
// capacity, world <= 8).  For token t and rank r holding one of its experts,
// the row goes to slot r*capacity + (number of earlier tokens that also go to
// r).  Tokens are taken 1024 at a time; per-rank running counts carry over.
// Outputs: per slot the source token (-1 for padding), per token pos[t][r] =
// slot or -1.  The metadata rows come from ep_meta_kernel (grid-wide).
constexpr int kEpPlanThreads = 1024;

__global__ void __launch_bounds__(kEpPlanThreads, 1)
ep_plan_fixed_kernel(const int32_t* __restrict__ ids, int m, int topk, int num_experts,
                     int world, int capacity, int64_t* __restrict__ send_src,
                     int64_t* __restrict__ pos) {
  __shared__ int warp_cnt[8][32];
  __shared__ int run[8];
  const int t0 = threadIdx.x;
  const int lane = t0 & 31, wid = t0 >> 5;
  const int e_loc = num_experts / world;
  if (t0 < 8) run[t0] = 0;
  __syncthreads();
  for (int base = 0; base < m; base += kEpPlanThreads) {
    const int t = base + t0;
    uint32_t has = 0;
    if (t < m) {
      for (int k = 0; k < topk; ++k) {
        const int e = ids[static_cast<int64_t>(t) * topk + k];
        if (e >= 0 && e < num_experts) has |= 1u << (e / e_loc);
      }
    }
    int rank_in[8];
    for (int r = 0; r < world; ++r) {
      const unsigned b = __ballot_sync(0xffffffffu, (has >> r) & 1u);
      rank_in[r] = __popc(b & ((1u << lane) - 1u));
      if (lane == 0) warp_cnt[r][wid] = __popc(b);
    }
    __syncthreads();
    if (t < m) {
      for (int r = 0; r < world; ++r) {
        int64_t slot = -1;
        if ((has >> r) & 1u) {
          int before = run[r];
          for (int q = 0; q < wid; ++q) before += warp_cnt[r][q];
          const int j = before + rank_in[r];
          slot = static_cast<int64_t>(r) * capacity + j;
          send_src[slot] = t;
        }
        pos[static_cast<int64_t>(t) * world + r] = slot;
      }
    }
    __syncthreads();
    if (t0 < world) {
      int tot = 0;
      for (int q = 0; q < 32; ++q) tot += warp_cnt[t0][q];
      run[t0] += tot;
    }
    __syncthreads();
  }
  // padding slots
  for (int r = 0; r < world; ++r)
    for (int j = run[r] + t0; j < capacity; j += kEpPlanThreads)
      send_src[static_cast<int64_t>(r) * capacity + j] = -1;
}

// Metadata rows of the fixed-capacity exchange, one thread per word, from the
// slot plan: slot s (rank r = s / capacity) of token t = send_src[s] gets
// {scale bits, local ids on r (-1 elsewhere), matching weights (0
// elsewhere)}; padding slots (t < 0) get {0, -1 x topk, 0 x topk}.  Rows sit
// meta_stride words apart.
__global__ void ep_meta_kernel(const int32_t* __restrict__ ids, const float* __restrict__ w,
                               const float* __restrict__ a_scale, int topk, int num_experts,
                               int world, int capacity, const int64_t* __restrict__ send_src,
                               int32_t* __restrict__ meta, int meta_words, int64_t meta_stride) {
  const int64_t total = static_cast<int64_t>(world) * capacity * meta_words;
  const int e_loc = num_experts / world;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t slot = i / meta_words;
    const int c = static_cast<int>(i - slot * meta_words);
    const int r = static_cast<int>(slot / capacity);
    const int64_t t = __ldg(send_src + slot);
    int32_t v = (c >= 1 && c <= topk) ? -1 : 0;
    if (t >= 0) {
      if (c == 0) {
        v = __float_as_int(__ldg(a_scale + t));
      } else if (c <= 2 * topk) {
        const int k = c <= topk ? c - 1 : c - 1 - topk;
        const int e = __ldg(ids + t * topk + k);
        const bool mine = e >= 0 && e < num_experts && e / e_loc == r;
        if (c <= topk) v = mine ? e - r * e_loc : -1;
        else v = __float_as_int(mine ? __ldg(w + t * topk + k) : 0.f);
      }
    }
    meta[slot * meta_stride + c] = v;
  }
}

// ---------------------------------------------------------------------------
// f2. Router top-k fused with the expert align: one cooperative launch from
// router logits to (topk_ids, topk_weights, sorted_token_ids, expert_ids,
// num_tokens_post_padded).  Same results, bit for bit, as router_topk_kernel
// followed by moe_align_kernel (stable order: increasing slot id inside each
// expert; padding value m*topk).  CTA c owns tokens [c*tpc, (c+1)*tpc) and its
// warps own contiguous sub-ranges, so slot order = (CTA, warp, token, k).
//   phase 1  route each token (router_row), count per (warp, expert) in
//            shared memory, publish per-(CTA, expert) totals; fill padding
//   grid sync
//   phase 2  per expert: CTA base (earlier CTAs' totals) and the
//            block-padded exclusive prefix over experts (every CTA computes
//            it); expert_ids / ntpp written grid-stride
//   phase 3  each warp places its slots
// Shared memory: wc [32][E] + cbase [E] + ebase [E + 1] + scan [32] ints.
// ---------------------------------------------------------------------------
constexpr int kRouteAlignThreads = 1024;

__host__ __device__ constexpr int route_align_smem_bytes(int experts) {
  return (32 * experts + experts + experts + 1 + 32) * 4;
}

template <typename T, int EPL>
__global__ void __launch_bounds__(kRouteAlignThreads, 1)
router_align_kernel(const T* __restrict__ logits, int m, int num_experts,
                    const float* __restrict__ bias, int topk, int renormalize, float scale,
                    int block_m, int tpc, int32_t* __restrict__ topk_ids,
                    float* __restrict__ topk_weights, int32_t* __restrict__ sorted_ids,
                    int sorted_cap, int32_t* __restrict__ expert_ids, int expert_cap,
                    int32_t* __restrict__ ntpp, int32_t* __restrict__ cta_counts,
                    int32_t* __restrict__ slot_pos) {
  extern __shared__ int sm_ra[];
  const int E = num_experts;
  int* wc = sm_ra;             // [32][E] per-warp counts, then per-warp cursors
  int* cbase = wc + 32 * E;    // [E] this CTA's base inside each expert
  int* ebase = cbase + E;      // [E + 1] padded exclusive prefix over experts
  int* scan = ebase + E + 1;   // [32]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, G = gridDim.x;
  const int t_begin = min(m, c * tpc), t_end = min(m, t_begin + tpc);
  const int tpw = (tpc + 31) / 32;
  const int w_begin = min(t_end, t_begin + warp * tpw), w_end = min(t_end, w_begin + tpw);
  const int numel = m * topk;

  for (int i = tid; i < 32 * E; i += kRouteAlignThreads) wc[i] = 0;
  for (int i = c * kRouteAlignThreads + tid; i < sorted_cap; i += G * kRouteAlignThreads)
    sorted_ids[i] = numel;
  __syncthreads();
  // phase 1: route, count
  for (int t = w_begin; t < w_end; ++t) {
    int id;
    float w;
    router_row<T, EPL>(logits, t, E, bias, topk, renormalize, scale, lane, id, w);
    if (lane < topk) {
      topk_ids[static_cast<int64_t>(t) * topk + lane] = id;
      topk_weights[static_cast<int64_t>(t) * topk + lane] = w;
      wc[warp * E + id] += 1;  // a token's experts are distinct: no two lanes collide
    }
    __syncwarp();
  }
  __syncthreads();
  for (int e = tid; e < E; e += kRouteAlignThreads) {
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int v = wc[w * E + e];
      wc[w * E + e] = run;
      run += v;
    }
    cta_counts[static_cast<int64_t>(c) * E + e] = run;
  }
  cooperative_groups::this_grid().sync();
  // phase 2: bases
  int cnt = 0;
  if (tid < E) {
    int before = 0, total = 0;
    for (int q = 0; q < G; ++q) {
      const int v = __ldcg(cta_counts + static_cast<int64_t>(q) * E + tid);
      if (q < c) before += v;
      total += v;
    }
    cbase[tid] = before;
    cnt = total;
  }
  {
    const int padded = (cnt + block_m - 1) / block_m * block_m;
    int v = padded;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += n;
    }
    if (lane == 31) scan[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int w = scan[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += n;
      }
      scan[lane] = w;
    }
    __syncthreads();
    const int incl = v + (warp > 0 ? scan[warp - 1] : 0);
    if (tid < E) ebase[tid] = incl - padded;
    if (tid == E - 1) ebase[E] = incl;
  }
  __syncthreads();
  const int total = ebase[E];
  for (int b = c * kRouteAlignThreads + tid; b < expert_cap; b += G * kRouteAlignThreads) {
    int e = -1;
    const int pos = b * block_m;
    if (pos < total) {
      int lo = 0, hi = E - 1;  // last e with ebase[e] <= pos
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (ebase[mid] <= pos) lo = mid; else hi = mid - 1;
      }
      e = lo;
    }
    expert_ids[b] = e;
  }
  if (c == 0 && tid == 0) ntpp[0] = total;
  // phase 3: place this warp's slots in (token, k) order
  for (int t = w_begin; t < w_end; ++t) {
    if (lane < topk) {
      const int e = topk_ids[static_cast<int64_t>(t) * topk + lane];
      const int pos = ebase[e] + cbase[e] + wc[warp * E + e];
      if (pos < sorted_cap) sorted_ids[pos] = t * topk + lane;
      if (slot_pos != nullptr) slot_pos[t * topk + lane] = pos < sorted_cap ? pos : -1;
      wc[warp * E + e] += 1;
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// a5, multi-CTA form (cooperative launch) for large inputs: the same outputs
// as moe_align_kernel, bit for bit.  CTA c owns flat ids [c*ipc, (c+1)*ipc),
// its warps contiguous sub-ranges, so (CTA, warp, index) is the slot order.
//   phase 1  per-(warp, expert) counts in shared memory (ids outside [0, E)
//            dropped), per-(CTA, expert) totals to `cta_counts`; padding fill
//   grid sync
//   phase 2  CTA base per expert, padded prefix over experts; expert_ids,
//            num_tokens_post_pad, cumsum
//   phase 3  placement, 32 ids at a time: __match_any groups equal experts,
//            the rank among lower lanes gives the position
// Shared memory: route_align_smem_bytes(E).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kRouteAlignThreads, 1)
moe_align_coop_kernel(const int32_t* __restrict__ ids, int numel, int num_experts, int block_m,
                      int ipc, int32_t* __restrict__ sorted_ids, int sorted_cap,
                      int32_t* __restrict__ expert_ids, int expert_cap,
                      int32_t* __restrict__ ntpp, int32_t* __restrict__ cumsum_out,
                      int32_t* __restrict__ cta_counts, int32_t* __restrict__ slot_pos) {
  extern __shared__ int sm_ac[];
  const int E = num_experts;
  int* wc = sm_ac;
  int* cbase = wc + 32 * E;
  int* ebase = cbase + E;
  int* scan = ebase + E + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, G = gridDim.x;
  const int i_begin = min(numel, c * ipc), i_end = min(numel, i_begin + ipc);
  const int ipw = (ipc + 31) / 32;
  const int w_begin = min(i_end, i_begin + warp * ipw), w_end = min(i_end, w_begin + ipw);

  for (int i = tid; i < 32 * E; i += kRouteAlignThreads) wc[i] = 0;
  for (int i = c * kRouteAlignThreads + tid; i < sorted_cap; i += G * kRouteAlignThreads)
    sorted_ids[i] = numel;
  __syncthreads();
  for (int i = w_begin + lane; i < w_end; i += 32) {
    const int e = __ldg(ids + i);
    if (e >= 0 && e < E) atomicAdd(&wc[warp * E + e], 1);
  }
  __syncthreads();
  for (int e = tid; e < E; e += kRouteAlignThreads) {
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int v = wc[w * E + e];
      wc[w * E + e] = run;
      run += v;
    }
    cta_counts[static_cast<int64_t>(c) * E + e] = run;
  }
  cooperative_groups::this_grid().sync();
  int cnt = 0;
  if (tid < E) {
    int before = 0, total = 0;
    for (int q = 0; q < G; ++q) {
      const int v = __ldcg(cta_counts + static_cast<int64_t>(q) * E + tid);
      if (q < c) before += v;
      total += v;
    }
    cbase[tid] = before;
    cnt = total;
  }
  {
    const int padded = (cnt + block_m - 1) / block_m * block_m;
    int v = padded;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += n;
    }
    if (lane == 31) scan[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int w = scan[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += n;
      }
      scan[lane] = w;
    }
    __syncthreads();
    const int incl = v + (warp > 0 ? scan[warp - 1] : 0);
    if (tid < E) ebase[tid] = incl - padded;
    if (tid == E - 1) ebase[E] = incl;
  }
  __syncthreads();
  const int total = ebase[E];
  for (int b = c * kRouteAlignThreads + tid; b < expert_cap; b += G * kRouteAlignThreads) {
    int e = -1;
    const int pos = b * block_m;
    if (pos < total) {
      int lo = 0, hi = E - 1;  // last e with ebase[e] <= pos
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (ebase[mid] <= pos) lo = mid; else hi = mid - 1;
      }
      e = lo;
    }
    expert_ids[b] = e;
  }
  if (c == 0) {
    if (tid == 0) ntpp[0] = total;
    if (cumsum_out != nullptr)
      for (int e = tid; e <= E; e += kRouteAlignThreads) cumsum_out[e] = ebase[e];
  }
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int i0 = w_begin; i0 < w_end; i0 += 32) {
    const int i = i0 + lane;
    const int e = i < w_end ? __ldg(ids + i) : -1;
    const bool valid = e >= 0 && e < E;
    const int key = valid ? e : (E + lane);  // unique key for invalid lanes
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int rank = __popc(peers & lt_mask);
    int pos = -1;
    if (valid) {
      pos = ebase[e] + cbase[e] + wc[warp * E + e] + rank;
      if (pos < sorted_cap) sorted_ids[pos] = i; else pos = -1;
    }
    if (slot_pos != nullptr && i < w_end) slot_pos[i] = pos;
    __syncwarp();
    if (valid && rank == 0) wc[warp * E + e] += __popc(peers);
    __syncwarp();
  }
}

// Dense split-K reduce: out = bf16((f32(sum_s partial) * a[m]) * cs[n])
// (reference DENSE_ENTRY:56-112).
__global__ void splitk_reduce_kernel(const int32_t* __restrict__ partial, int splits,
                                     int64_t split_stride, int64_t ld,
                                     const float* __restrict__ a_scale,
                                     const float* __restrict__ cs, __nv_bfloat16* __restrict__ out,
                                     int m, int n) {
  pdl_entry();
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(m) * n) return;
  const int row = static_cast<int>(idx / n);
  const int col = static_cast<int>(idx - static_cast<int64_t>(row) * n);
  int32_t acc = 0;
  for (int s = 0; s < splits; ++s) acc += __ldg(partial + s * split_stride + row * ld + col);
  const float v = __fmul_rn(__fmul_rn(__int2float_rn(acc), __ldg(a_scale + row)), __ldg(cs + col));
  out[idx] = __float2bfloat16_rn(v);
}

}  // namespace dsv4
