// C ABI of the B200 MXFP4/INT8 MoE path (declared in include/dsv4_b200.h).
// Single translation unit: the device status word and every kernel live here.

#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdlib>
#include <utility>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "small_kernels.cuh"

namespace dsv4 {

namespace {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DSV4_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return DSV4_OK;
}

#define DSV4_REQUIRE(cond, ...) \
  do {                          \
    if (!(cond)) return fail(DSV4_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Kernels of the hot path are launched with programmatic stream
// serialisation (each calls pdl_entry() before touching global memory), so a
// kernel's launch and scheduling overlap its predecessor's tail.
// DSV4_B200_PDL=0 turns the attribute off.
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("DSV4_B200_PDL");
    return e == nullptr || std::strcmp(e, "0") != 0;
  }();
  return on;
}

template <typename... KArgs, typename... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  // errors surface through cudaGetLastError in check_launch
  (void)cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Cluster-of-2 launch (CTA pairs of the 2-SM MMA), with programmatic
// dependent launch as launch_pdl.
template <typename... KArgs, typename... Args>
void launch_pair(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                 Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  (void)cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// 256-token tiles run on CTA pairs only with DSV4_B200_PAIR=1 (read at each
// launch, so one process can compare both forms).  Off by default: measured
// slower than single CTAs (prefill 4.06 vs 3.32 ms) — the cross-SM hand-off
// of every stage (remote cluster-scope arrivals) is not hidden by the 2-slot
// A ring that the TMEM stash leaves.
bool pair_enabled() {
  const char* e = std::getenv("DSV4_B200_PAIR");
  return e != nullptr && std::strcmp(e, "1") == 0;
}

constexpr int kMaxDevices = 64;
std::mutex g_init_mu;
bool g_inited[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};

template <int TN, int EPI>
struct GemmKernel {
  static constexpr int kSmem = TcGemmCfg<TN, (EPI & kEpiPair) != 0>::kSmemLaunch;
  static void* fn() { return reinterpret_cast<void*>(&mxfp4_int8_tc_gemm_kernel<TN, EPI>); }
};

template <int EPI>
cudaError_t set_attrs_epi() {
  cudaError_t e = cudaSuccess;
  auto one = [&](void* f, int smem) {
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  };
  one(GemmKernel<16, EPI>::fn(), GemmKernel<16, EPI>::kSmem);
  one(GemmKernel<32, EPI>::fn(), GemmKernel<32, EPI>::kSmem);
  one(GemmKernel<64, EPI>::fn(), GemmKernel<64, EPI>::kSmem);
  one(GemmKernel<128, EPI>::fn(), GemmKernel<128, EPI>::kSmem);
  one(GemmKernel<192, EPI>::fn(), GemmKernel<192, EPI>::kSmem);
  one(GemmKernel<256, EPI>::fn(), GemmKernel<256, EPI>::kSmem);
  return e;
}

constexpr int kAlignMaxExperts = 1024;
int align_smem_bytes(int experts) { return (32 * experts + experts + 1 + 32) * 4; }

cudaError_t set_router_align_attrs();

int ensure_init() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(DSV4_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(DSV4_ERR_CUDA, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_init_mu);
  if (g_inited[dev]) return DSV4_OK;
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0)
    return fail(DSV4_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
                dev, major, minor);
  e = set_attrs_epi<kEpiBf16>();
  if (e == cudaSuccess) e = set_attrs_epi<kEpiI32>();
  if (e == cudaSuccess) e = set_attrs_epi<kEpiSwiglu>();
  if (e == cudaSuccess) e = set_attrs_epi<kEpiBf16 | kEpiBiased>();
  if (e == cudaSuccess) e = set_attrs_epi<kEpiSwiglu | kEpiBiased>();
  // CTA-pair instantiations exist for 256-token tiles only
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(GemmKernel<256, kEpiBf16 | kEpiBiased | kEpiPair>::fn(),
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             GemmKernel<256, kEpiBf16 | kEpiBiased | kEpiPair>::kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(GemmKernel<256, kEpiSwiglu | kEpiBiased | kEpiPair>::fn(),
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             GemmKernel<256, kEpiSwiglu | kEpiBiased | kEpiPair>::kSmem);
  if (e == cudaSuccess) e = set_router_align_attrs();
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(reinterpret_cast<void*>(&moe_align_kernel),
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             align_smem_bytes(kAlignMaxExperts));
  if (e != cudaSuccess)
    return fail(DSV4_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  cudaDeviceGetAttribute(&g_sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
  g_inited[dev] = true;
  return DSV4_OK;
}

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  return g_sm_count[dev] > 0 ? g_sm_count[dev] : 148;
}

// Persistent launch of CTA pairs: one pair per two SMs, never more pairs than
// pair items (an item = one token tile x two neighbouring row tiles).
template <int EPI>
int launch_gemm_pair(int64_t max_pair_items, const TcGemmParams& p, cudaStream_t st) {
  int64_t pairs = sm_count() / 2;
  if (max_pair_items < pairs) pairs = max_pair_items;
  if (pairs <= 0) return DSV4_OK;
  const dim3 grid(static_cast<unsigned>(2 * pairs));
  constexpr int kE = EPI | kEpiPair;
  launch_pair(&mxfp4_int8_tc_gemm_kernel<256, kE>, grid, TcGemmCfg<256, true>::kThreads,
              GemmKernel<256, kE>::kSmem, st, p);
  return check_launch("mxfp4_int8_tc_gemm_kernel (CTA pairs)");
}

// Persistent launch: one CTA per SM (never more CTAs than work items).
template <int EPI>
int launch_gemm(int tn, int64_t max_items, const TcGemmParams& p, cudaStream_t st) {
  const int64_t ctas = max_items < sm_count() ? max_items : sm_count();
  if (ctas <= 0) return DSV4_OK;
  const dim3 grid(static_cast<unsigned>(ctas));
  switch (tn) {
#define DSV4_CASE(T)                                                                    \
  case T:                                                                               \
    launch_pdl(&mxfp4_int8_tc_gemm_kernel<T, EPI>, grid, TcGemmCfg<T>::kThreads, GemmKernel<T, EPI>::kSmem, st, p); \
    break;
    DSV4_CASE(16)
    DSV4_CASE(32)
    DSV4_CASE(64)
    DSV4_CASE(128)
    DSV4_CASE(192)
    DSV4_CASE(256)
#undef DSV4_CASE
    default:
      return fail(DSV4_ERR_INVALID_ARGUMENT, "unsupported token tile %d", tn);
  }
  return check_launch("mxfp4_int8_tc_gemm_kernel");
}

// ---- tensor maps for the weight stream (driver entry point, no -lcuda) ----
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

CUresult encode_u8(CUtensorMap* map, int rank, const void* base, const cuuint64_t* dims,
                   const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle swz,
                   CUtensorMapL2promotion l2) {
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return tensor_map_encoder()(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, const_cast<void*>(base),
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, l2,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// Weight maps, one box per 256-K stage and one shift box per chunk of
// kShChunk stages (sh_rows = 2 shift rows per stage, <= 2 * kShChunk):
//   plain   b_mxfp4 [E][KB][NG8][128] as 3-D {128, NG8, E*KB}, box {128, 16, 8};
//           b_shift2 [E][SS][N] as 2-D {N, E*SS}, box {128, sh_rows}
//   SwiGLU  the gate rows [0, I) and up rows [I, 2I) as a plane dimension:
//           b_mxfp4 as 4-D {128, I/8, 2, E*KB}, box {128, 8, 2, 8};
//           b_shift2 as 3-D {I, 2, E*SS}, box {64, 2, sh_rows}
int encode_weight_maps(TcGemmParams& p, const uint8_t* b_mxfp4, const uint8_t* b_shift2,
                       int64_t experts, int64_t kb, int64_t ss, int64_t ng8, bool swiglu,
                       int64_t inter, int sh_rows) {
  if (tensor_map_encoder() == nullptr) return fail(DSV4_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  DSV4_REQUIRE((reinterpret_cast<uintptr_t>(b_mxfp4) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(b_shift2) & 15) == 0,
               "weight tensors must be 16-byte aligned");
  DSV4_REQUIRE(experts * kb < (1ll << 31) && experts * ss < (1ll << 31), "weight too large");
  DSV4_REQUIRE(sh_rows >= 2 && sh_rows <= 2 * TcGemmCfg<16>::kShChunk, "bad shift chunk");
  const cuuint64_t n = static_cast<cuuint64_t>(ng8 * 8);
  CUresult r;
  if (swiglu) {
    DSV4_REQUIRE(inter % 64 == 0 && 2 * inter == ng8 * 8, "SwiGLU needs N = 2 * I, I % 64 == 0");
    const cuuint64_t i = static_cast<cuuint64_t>(inter);
    cuuint64_t dims[4] = {128, i / 8, 2, static_cast<cuuint64_t>(experts * kb)};
    cuuint64_t strides[3] = {128, i * 16, n * 16};
    cuuint32_t box[4] = {128, 8, 2, 8};
    r = encode_u8(&p.map_packed, 4, b_mxfp4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  } else {
    cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(ng8), static_cast<cuuint64_t>(experts * kb)};
    cuuint64_t strides[2] = {128, n * 16};
    cuuint32_t box[3] = {128, 16, 8};
    r = encode_u8(&p.map_packed, 3, b_mxfp4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  }
  if (r != CUDA_SUCCESS) return fail(DSV4_ERR_CUDA, "tensor map (packed) encode failed: %d", (int)r);
  if (swiglu) {
    const cuuint64_t i = static_cast<cuuint64_t>(inter);
    cuuint64_t dims[3] = {i, 2, static_cast<cuuint64_t>(experts * ss)};
    cuuint64_t strides[2] = {i, n};
    cuuint32_t box[3] = {64, 2, static_cast<cuuint32_t>(sh_rows)};
    r = encode_u8(&p.map_shift, 3, b_shift2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE);
  } else {
    cuuint64_t dims[2] = {n, static_cast<cuuint64_t>(experts * ss)};
    cuuint64_t strides[1] = {n};
    cuuint32_t box[2] = {128, static_cast<cuuint32_t>(sh_rows)};
    r = encode_u8(&p.map_shift, 2, b_shift2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE);
  }
  if (r != CUDA_SUCCESS) return fail(DSV4_ERR_CUDA, "tensor map (shift) encode failed: %d", (int)r);
  p.kb_per_expert = static_cast<int>(kb);
  p.ss_per_expert = static_cast<int>(ss);
  p.sh_rows = sh_rows;
  return DSV4_OK;
}

int shift_chunk_rows(int stages_per_item, int tn) {
  const int c = tn >= 256 ? TcGemmCfg<256>::kShChunk : TcGemmCfg<16>::kShChunk;
  return 2 * (stages_per_item < c ? stages_per_item : c);
}

// Activation (B operand) maps, all with the 128-byte swizzle of the K-major
// SW128 MMA layout:
//   b_mode 0: int8 [rows][k] as 2-D {k, rows}, box {128, 1} (tile::gather4)
//   b_mode 1: int8 [rows][k] as 2-D {k, rows}, box {128, tn}
//   b_mode 2: int8 K-chunk-major [k/128][rows][128] as 3-D {128, rows, k/128},
//             box {128, tn, 2} (both 128-K halves of a stage in one copy)
int encode_act_map(TcGemmParams& p, const int8_t* a, int64_t rows, int64_t k, int b_mode, int tn,
                   bool pair = false) {
  DSV4_REQUIRE(tn <= 128 || b_mode == 2, "192/256-token tiles need K-chunk-major token rows");
  if (tensor_map_encoder() == nullptr) return fail(DSV4_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  DSV4_REQUIRE((reinterpret_cast<uintptr_t>(a) & 15) == 0, "a_q must be 16-byte aligned");
  DSV4_REQUIRE(rows >= 1 && rows < (1ll << 31), "bad activation row count");
  CUresult r;
  if (b_mode == 2) {
    DSV4_REQUIRE(k % 128 == 0, "K-chunk-major rows need K %% 128 == 0");
    cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(k / 128)};
    cuuint64_t strides[2] = {128, static_cast<cuuint64_t>(rows) * 128};
    // CTA pairs: each CTA stages half of the token tile
    cuuint32_t box[3] = {128, static_cast<cuuint32_t>(pair ? tn / 2 : tn), 2};
    r = encode_u8(&p.map_act, 3, a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    p.short_rows = 0;
    if (r == CUDA_SUCCESS && !pair && tn > 64) {
      // 64-row box of one 128-K half, for blocks with at most 64 tokens (MoE
      // remainder blocks); a stage takes two, one into each half of its slot
      cuuint32_t sbox[3] = {128, 64, 1};
      r = encode_u8(&p.map_act_short, 3, a, dims, strides, sbox, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
      p.short_rows = 64;
    }
  } else {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(k)};
    cuuint32_t box[2] = {128, static_cast<cuuint32_t>(b_mode == 1 ? tn : 1)};
    r = encode_u8(&p.map_act, 2, a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  }
  if (r != CUDA_SUCCESS) return fail(DSV4_ERR_CUDA, "tensor map (activations) encode failed: %d", (int)r);
  p.b_mode = b_mode;
  return DSV4_OK;
}

int64_t align_capacity(int64_t numel, int64_t experts, int64_t bm) {
  return numel < experts + 1 ? numel * bm : numel + (experts + 1) * (bm - 1);
}

int check_weights(int64_t experts, int64_t n, int64_t k, int64_t shift_stride) {
  DSV4_REQUIRE(experts >= 1, "num_experts must be >= 1, got %lld", (long long)experts);
  DSV4_REQUIRE(n > 0 && n % 128 == 0, "N must be a positive multiple of 128, got %lld",
               (long long)n);
  DSV4_REQUIRE(k > 0 && k % 128 == 0, "K must be divisible by 128, got %lld", (long long)k);
  DSV4_REQUIRE(shift_stride >= (k / 32 + 3) / 4, "b_shift2 stride mismatch (%lld < %lld)",
               (long long)shift_stride, (long long)((k / 32 + 3) / 4));
  return DSV4_OK;
}

int moe_gemm_common(int epi, const int8_t* a_q, const float* a_scale, int64_t m_in,
                    const uint8_t* b_mxfp4, const uint8_t* b_shift2, const float* cs,
                    int64_t experts, int64_t n_rows, int64_t k, int64_t shift_stride, void* dst,
                    int64_t ldo, int64_t tile_rows_y, int64_t inter,
                    const int32_t* sorted_ids, int64_t sorted_cap, const int32_t* expert_ids,
                    int64_t expert_cap, const int32_t* ntpp, int64_t topk, int64_t block_m,
                    int src_is_slot, int64_t num_valid, int has_clamp, float clamp_limit,
                    void* stream, bool sorted_rows = false,
                    const int32_t* a_rowsum = nullptr) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(a_q && a_scale && b_mxfp4 && b_shift2 && cs && dst && sorted_ids && expert_ids &&
                   ntpp,
               "null pointer argument");
  if (int r = check_weights(experts, n_rows, k, shift_stride)) return r;
  DSV4_REQUIRE((reinterpret_cast<uintptr_t>(cs) & 15) == 0, "b_channel_scale must be 16-byte aligned");
  DSV4_REQUIRE((reinterpret_cast<uintptr_t>(dst) & 15) == 0, "output must be 16-byte aligned");
  DSV4_REQUIRE(topk >= 1 && topk <= 8, "topk must be in [1, 8], got %lld", (long long)topk);
  DSV4_REQUIRE(block_m == 16 || block_m == 32 || block_m == 64 || block_m == 128 ||
                   (sorted_rows && (block_m == 192 || block_m == 256)),
               "block_m must be 16, 32, 64, or 128 (or 192 / 256 for sorted rows), got %lld",
               (long long)block_m);
  DSV4_REQUIRE(num_valid >= 0, "num_valid_tokens must be non-negative");
  const int64_t max_m = align_capacity(num_valid, experts, block_m);
  if (sorted_rows) DSV4_REQUIRE(a_rowsum != nullptr, "a_rowsum is null");
  if (sorted_rows)
    DSV4_REQUIRE(m_in == sorted_cap, "sorted input rows (%lld) must equal the sorted_token_ids "
                 "capacity (%lld)", (long long)m_in, (long long)sorted_cap);
  else if (src_is_slot)
    DSV4_REQUIRE(m_in >= num_valid, "W2 input rows do not cover routed slots");
  else
    DSV4_REQUIRE(m_in * topk >= num_valid, "W13 input rows do not cover routed slots");
  const int64_t grid_m = (max_m + block_m - 1) / block_m;
  DSV4_REQUIRE(sorted_cap >= max_m,
               "sorted_token_ids capacity is smaller than maximum aligned token count");
  DSV4_REQUIRE(expert_cap >= grid_m, "expert_ids capacity is smaller than maximum M tile count");
  if (num_valid == 0 || grid_m == 0) return DSV4_OK;
  DSV4_REQUIRE(grid_m <= 0x7FFFFFFF, "too many M tiles");

  TcGemmParams p{};
  p.dec_m1 = 0xFFFFFFFFu;
  p.dec_hi16 = 65536u;
  p.dec_one = 1u;
  p.a = a_q;
  p.a_scale = a_scale;
  p.a_rowsum = a_rowsum;
  p.lda = k;
  p.a_rows = m_in;
  p.cs = cs;
  p.n = static_cast<int>(n_rows);
  p.inter = static_cast<int>(inter);
  p.k_stages = static_cast<int>((k / 32 + 7) / 8);  // 256-K stages
  p.stages_per_split = p.k_stages;
  p.splits = 1;
  p.row_tiles = static_cast<int>(tile_rows_y);
  p.moe = 1;
  p.sorted_ids = sorted_ids;
  p.expert_ids = expert_ids;
  p.ntpp = ntpp;
  p.block_m = static_cast<int>(block_m);
  p.topk = static_cast<int>(topk);
  p.num_valid = static_cast<int>(num_valid);
  p.src_is_slot = src_is_slot;
  p.a_row_mode = sorted_rows ? 2 : (src_is_slot ? 1 : 0);
  p.out_sorted = sorted_rows && epi == kEpiSwiglu ? 1 : 0;
  p.out = reinterpret_cast<__nv_bfloat16*>(dst);
  p.ldo = ldo;
  p.has_clamp = has_clamp;
  p.clamp_limit = clamp_limit;
  if (int r = encode_weight_maps(p, b_mxfp4, b_shift2, experts, k / 32, shift_stride, n_rows / 8,
                                 epi == kEpiSwiglu, inter, shift_chunk_rows(p.k_stages, static_cast<int>(block_m))))
    return r;
  // 256-token tiles of the sorted path: CTA pairs (each CTA its own row tile
  // of a neighbouring pair, half of the token tile)
  const bool pair = pair_enabled() && block_m == 256 && sorted_rows && a_rowsum != nullptr &&
                    tile_rows_y % 2 == 0;
  if (int r = encode_act_map(p, a_q, m_in, k, sorted_rows ? 2 : 0, static_cast<int>(block_m), pair))
    return r;
  const int64_t max_items = grid_m * tile_rows_y;
  const int bm = static_cast<int>(block_m);
  if (pair) {
    if (epi == kEpiSwiglu)
      return launch_gemm_pair<kEpiSwiglu | kEpiBiased>(max_items / 2, p, as_stream(stream));
    return launch_gemm_pair<kEpiBf16 | kEpiBiased>(max_items / 2, p, as_stream(stream));
  }
  if (a_rowsum != nullptr) {  // biased-unsigned decode, corrected by the row sums
    if (epi == kEpiSwiglu)
      return launch_gemm<kEpiSwiglu | kEpiBiased>(bm, max_items, p, as_stream(stream));
    return launch_gemm<kEpiBf16 | kEpiBiased>(bm, max_items, p, as_stream(stream));
  }
  if (epi == kEpiSwiglu) return launch_gemm<kEpiSwiglu>(bm, max_items, p, as_stream(stream));
  return launch_gemm<kEpiBf16>(bm, max_items, p, as_stream(stream));
}

int dense_tile(int64_t m) {
  if (m <= 16) return 16;
  if (m <= 32) return 32;
  if (m <= 64) return 64;
  return 128;
}

int dense_common(const int8_t* a_q, const float* a_scale, int64_t m, int64_t k,
                 const uint8_t* b_mxfp4, const uint8_t* b_shift2, int64_t shift_stride,
                 const float* cs, int64_t n, void* out, int32_t* out_i32, int64_t splits,
                 int64_t ld, int64_t split_stride, int epi, void* stream,
                 const int32_t* a_rowsum = nullptr) {
  // a_rowsum set: activations are K-chunk-major [K/128][m][128] with int8 row
  // sums, 256-token tiles, biased-unsigned decode (the expert-sorted path's
  // tile, with one "expert")
  if (int r = check_weights(1, n, k, shift_stride)) return r;
  DSV4_REQUIRE(cs == nullptr || (reinterpret_cast<uintptr_t>(cs) & 15) == 0,
               "weight_channel_scale must be 16-byte aligned");
  DSV4_REQUIRE(out == nullptr || (reinterpret_cast<uintptr_t>(out) & 15) == 0,
               "out must be 16-byte aligned");
  TcGemmParams p{};
  p.dec_m1 = 0xFFFFFFFFu;
  p.dec_hi16 = 65536u;
  p.dec_one = 1u;
  p.a = a_q;
  p.a_scale = a_scale;
  p.a_rowsum = a_rowsum;
  p.lda = k;
  p.a_rows = m;
  p.cs = cs;
  p.n = static_cast<int>(n);
  p.k_stages = static_cast<int>((k / 32 + 7) / 8);  // 256-K stages
  p.stages_per_split = static_cast<int>((p.k_stages + splits - 1) / splits);
  p.splits = static_cast<int>((p.k_stages + p.stages_per_split - 1) / p.stages_per_split);
  p.moe = 0;
  p.m = static_cast<int>(m);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.out_i32 = out_i32;
  p.ldo = ld;
  p.split_stride = split_stride;
  const bool cm = a_rowsum != nullptr;
  const int tn = cm ? 256 : dense_tile(m);
  if (int r = encode_weight_maps(p, b_mxfp4, b_shift2, 1, k / 32, shift_stride, n / 8, false, 0,
                                 shift_chunk_rows(p.stages_per_split, tn)))
    return r;
  const bool pair = cm && pair_enabled() && (n / 128) % 2 == 0;
  if (int r = encode_act_map(p, a_q, m, k, cm ? 2 : 1, tn, pair)) return r;
  p.m_tiles = static_cast<int>((m + tn - 1) / tn);
  p.row_tiles = static_cast<int>(n / 128);
  const int64_t max_items = static_cast<int64_t>(p.m_tiles) * p.row_tiles * p.splits;
  if (pair) return launch_gemm_pair<kEpiBf16 | kEpiBiased>(max_items / 2, p, as_stream(stream));
  if (cm) return launch_gemm<kEpiBf16 | kEpiBiased>(tn, max_items, p, as_stream(stream));
  if (epi == kEpiI32) return launch_gemm<kEpiI32>(tn, max_items, p, as_stream(stream));
  return launch_gemm<kEpiBf16>(tn, max_items, p, as_stream(stream));
}

// ---- fused router + align (cooperative launch) ----
template <typename T>
const void* router_align_fn_t(int epl) {
  if (epl <= 1) return reinterpret_cast<const void*>(&router_align_kernel<T, 1>);
  if (epl <= 2) return reinterpret_cast<const void*>(&router_align_kernel<T, 2>);
  if (epl <= 4) return reinterpret_cast<const void*>(&router_align_kernel<T, 4>);
  if (epl <= 8) return reinterpret_cast<const void*>(&router_align_kernel<T, 8>);
  if (epl <= 16) return reinterpret_cast<const void*>(&router_align_kernel<T, 16>);
  return reinterpret_cast<const void*>(&router_align_kernel<T, 32>);
}

const void* router_align_fn(int dtype, int epl) {
  switch (dtype) {
    case DSV4_F32: return router_align_fn_t<float>(epl);
    case DSV4_F16: return router_align_fn_t<__half>(epl);
    case DSV4_BF16: return router_align_fn_t<__nv_bfloat16>(epl);
    default: return nullptr;
  }
}

cudaError_t set_router_align_attrs() {
  cudaError_t e = cudaSuccess;
  for (int dt : {DSV4_F32, DSV4_F16, DSV4_BF16})
    for (int epl : {1, 2, 4, 8, 16, 32})
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(router_align_fn(dt, epl),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 route_align_smem_bytes(kAlignMaxExperts));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&moe_align_coop_kernel),
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             route_align_smem_bytes(kAlignMaxExperts));
  return e;
}

// CTAs of the multi-CTA align: about 1,024 ids each, at most one per SM.
int64_t align_coop_grid(int64_t numel) {
  int64_t g = (numel + 1023) / 1024;
  if (g < 1) g = 1;
  return g < sm_count() ? g : sm_count();
}

// CTAs of the fused router + align: one per 64 tokens, at most one per SM
// (co-resident, as the grid-wide barrier needs).
int64_t router_align_grid(int64_t m) {
  int64_t g = (m + 63) / 64;
  if (g < 1) g = 1;
  return g < sm_count() ? g : sm_count();
}

// Fixed split-K workspace of dsv4_b200_mxfp4_int8_dense_gemm_noalloc:
// 4 splits x 128 rows x 4096 columns of int32 (8 MiB) per device that loads
// the library, held until process exit.  In host code `g_noalloc_splitk` is
// only a stand-in symbol; the kernels get the address from
// cudaGetSymbolAddress (noalloc_scratch()).
constexpr int64_t kNoAllocScratchWords = 4ll * 128 * 4096;
static __device__ __align__(256) int32_t g_noalloc_splitk[kNoAllocScratchWords];
int32_t* g_noalloc_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

int noalloc_scratch(int32_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(DSV4_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_splitk);
    if (e != cudaSuccess || p == nullptr)
      return fail(DSV4_ERR_CUDA, "cudaGetSymbolAddress(split-K workspace): %s",
                  cudaGetErrorString(e));
    g_noalloc_ptr[dev] = static_cast<int32_t*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return DSV4_OK;
}

}  // namespace
}  // namespace dsv4

using namespace dsv4;

extern "C" {

int dsv4_b200_abi_version(void) { return DSV4_B200_ABI_VERSION; }

const char* dsv4_b200_last_error(void) { return g_last_error; }

int dsv4_b200_init(int device) {
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return fail(DSV4_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (device != prev) {
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return fail(DSV4_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
  }
  int r = ensure_init();
  if (device != prev) cudaSetDevice(prev);
  return r;
}

int dsv4_b200_get_device_status(int* status, int reset) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(status != nullptr, "status is null");
  cudaError_t e = cudaMemcpyFromSymbol(status, g_device_status, sizeof(int));
  if (e != cudaSuccess) return fail(DSV4_ERR_CUDA, "read status: %s", cudaGetErrorString(e));
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
    if (e != cudaSuccess) return fail(DSV4_ERR_CUDA, "reset status: %s", cudaGetErrorString(e));
  }
  return DSV4_OK;
}

int dsv4_b200_quantize_per_token_int8(const void* a, int dtype, int64_t m, int64_t k, int64_t lda,
                                      float clamp_abs, int8_t* a_q, float* a_scale,
                                      void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(m >= 0 && k >= 0 && lda >= k, "bad shape m=%lld k=%lld lda=%lld", (long long)m,
               (long long)k, (long long)lda);
  if (m == 0) return DSV4_OK;
  DSV4_REQUIRE(a && a_q && a_scale, "null pointer argument");
  cudaStream_t st = as_stream(stream);
  const bool reg_ok = (dtype == DSV4_F16 || dtype == DSV4_BF16) && k % 8 == 0 && lda % 8 == 0 &&
                      (reinterpret_cast<uintptr_t>(a) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(a_q) & 7) == 0 && k <= 8192;
  if (reg_ok) {
    // register-resident rows: 128 threads per row for long rows, a warp otherwise
    const bool wide = k > 2048;
    const int rows_per_cta = wide ? 2 : 8;
    const dim3 g(static_cast<unsigned>((m + rows_per_cta - 1) / rows_per_cta));
    if (dtype == DSV4_BF16) {
      if (wide) launch_pdl(&quant_rows_reg_kernel<__nv_bfloat16, 128, 8>, g, 256, 0, st, static_cast<const __nv_bfloat16*>(a), m, k, lda, clamp_abs, a_q, a_scale, nullptr, nullptr, 0, 0, nullptr, 0);
      else launch_pdl(&quant_rows_reg_kernel<__nv_bfloat16, 32, 8>, g, 256, 0, st, static_cast<const __nv_bfloat16*>(a), m, k, lda, clamp_abs, a_q, a_scale, nullptr, nullptr, 0, 0, nullptr, 0);
    } else {
      if (wide) launch_pdl(&quant_rows_reg_kernel<__half, 128, 8>, g, 256, 0, st, static_cast<const __half*>(a), m, k, lda, clamp_abs, a_q, a_scale, nullptr, nullptr, 0, 0, nullptr, 0);
      else launch_pdl(&quant_rows_reg_kernel<__half, 32, 8>, g, 256, 0, st, static_cast<const __half*>(a), m, k, lda, clamp_abs, a_q, a_scale, nullptr, nullptr, 0, 0, nullptr, 0);
    }
    return check_launch("quant_rows_reg_kernel");
  }
  const dim3 grid(static_cast<unsigned>((m + 7) / 8));
  switch (dtype) {
    case DSV4_F32:
      launch_pdl(&quant_rows_kernel<float>, grid, 256, 0, st, static_cast<const float*>(a), m, k, lda,
                                                     clamp_abs, a_q, a_scale);
      break;
    case DSV4_F16:
      launch_pdl(&quant_rows_kernel<__half>, grid, 256, 0, st, static_cast<const __half*>(a), m, k, lda,
                                                      clamp_abs, a_q, a_scale);
      break;
    case DSV4_BF16:
      launch_pdl(&quant_rows_kernel<__nv_bfloat16>, grid, 256, 0, st, 
          static_cast<const __nv_bfloat16*>(a), m, k, lda, clamp_abs, a_q, a_scale);
      break;
    default:
      return fail(DSV4_ERR_INVALID_ARGUMENT, "a must be fp32, fp16, or bf16 (dtype %d)", dtype);
  }
  return check_launch("quant_rows_kernel");
}

int dsv4_b200_remap_mxfp4_weight_for_int8(const uint8_t* weight, const uint8_t* scale,
                                          int64_t experts, int64_t n, int64_t k,
                                          int headroom_bits, int round_half_even,
                                          uint8_t* b_mxfp4, uint8_t* b_shift2,
                                          float* channel_scale, void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(headroom_bits >= 0 && headroom_bits <= 7, "invalid headroom_bits=%d",
               headroom_bits);
  DSV4_REQUIRE(experts >= 0 && n >= 0 && k >= 0 && k % 32 == 0,
               "expected K divisible by 32, got %lld", (long long)k);
  if (experts == 0 || n == 0 || k == 0) return DSV4_OK;
  DSV4_REQUIRE(weight && scale && b_mxfp4 && b_shift2 && channel_scale, "null pointer argument");
  const int kb = static_cast<int>(k / 32);
  const int ss = (kb + 3) / 4;
  const int ng8 = static_cast<int>((n + 7) / 8);
  cudaStream_t st = as_stream(stream);
  // pad rows of the last 8-row group must read as zero
  if (n % 8 != 0) {
    cudaError_t e = cudaMemsetAsync(b_shift2, 0, experts * ss * ng8 * 8, st);
    if (e != cudaSuccess) return fail(DSV4_ERR_CUDA, "memset: %s", cudaGetErrorString(e));
  }
  const int64_t rows = experts * n;
  repack_channel_shift_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, st>>>(
      scale, rows, static_cast<int>(n), kb, ss, ng8, headroom_bits, channel_scale, b_shift2);
  if (int r = check_launch("repack_channel_shift_kernel")) return r;
  const int64_t words = experts * kb * ng8 * 32;
  repack_codes_kernel<<<static_cast<unsigned>((words + 255) / 256), 256, 0, st>>>(
      weight, scale, channel_scale, words, static_cast<int>(n), kb, ng8, headroom_bits,
      round_half_even, reinterpret_cast<uint32_t*>(b_mxfp4));
  return check_launch("repack_codes_kernel");
}

int dsv4_b200_router_topk(const void* logits, int dtype, int64_t m, int64_t num_experts,
                          const float* bias, int64_t topk, int renormalize, float scale,
                          int32_t* topk_ids, float* topk_weights, void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(m >= 0 && m < (1ll << 31), "bad m %lld", (long long)m);
  DSV4_REQUIRE(num_experts >= 1 && num_experts <= 1024, "num_experts must be in [1, 1024]");
  DSV4_REQUIRE(topk >= 1 && topk <= 32 && topk <= num_experts, "topk must be in [1, min(32, E)]");
  if (m == 0) return DSV4_OK;
  DSV4_REQUIRE(logits && topk_ids && topk_weights, "null pointer argument");
  const int epl = static_cast<int>((num_experts + 31) / 32);
  const dim3 grid(static_cast<unsigned>((m + 7) / 8));
  cudaStream_t st = as_stream(stream);
  const int e = static_cast<int>(num_experts), k = static_cast<int>(topk);
#define DSV4_RT(T, EPL)                                                                       \
  router_topk_kernel<T, EPL><<<grid, 256, 0, st>>>(static_cast<const T*>(logits), m, e, bias, k, \
                                                   renormalize, scale, topk_ids, topk_weights)
#define DSV4_RT_E(T)                                    \
  if (epl <= 1) DSV4_RT(T, 1);                          \
  else if (epl <= 2) DSV4_RT(T, 2);                     \
  else if (epl <= 4) DSV4_RT(T, 4);                     \
  else if (epl <= 8) DSV4_RT(T, 8);                     \
  else if (epl <= 16) DSV4_RT(T, 16);                   \
  else DSV4_RT(T, 32)
  switch (dtype) {
    case DSV4_F32: DSV4_RT_E(float); break;
    case DSV4_F16: DSV4_RT_E(__half); break;
    case DSV4_BF16: DSV4_RT_E(__nv_bfloat16); break;
    default:
      return fail(DSV4_ERR_INVALID_ARGUMENT, "logits must be fp32, fp16, or bf16 (dtype %d)", dtype);
  }
#undef DSV4_RT_E
#undef DSV4_RT
  return check_launch("router_topk_kernel");
}

int dsv4_b200_router_align_workspace_words(int64_t m, int64_t num_experts, int64_t* words) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(words != nullptr && m >= 0 && num_experts >= 1, "bad arguments");
  *words = router_align_grid(m) * num_experts;
  return DSV4_OK;
}

int dsv4_b200_router_align(const void* logits, int dtype, int64_t m, int64_t num_experts,
                           const float* bias, int64_t topk, int renormalize, float scale,
                           int64_t block_size, int32_t* topk_ids, float* topk_weights,
                           int32_t* sorted_token_ids, int64_t sorted_capacity,
                           int32_t* expert_ids, int64_t expert_ids_capacity,
                           int32_t* num_tokens_post_pad, int32_t* workspace,
                           int64_t workspace_words, int32_t* slot_pos, void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(m >= 0 && m < (1ll << 27), "bad m %lld", (long long)m);
  DSV4_REQUIRE(num_experts >= 1 && num_experts <= kAlignMaxExperts,
               "num_experts must be in [1, %d]", kAlignMaxExperts);
  DSV4_REQUIRE(topk >= 1 && topk <= 32 && topk <= num_experts, "topk must be in [1, min(32, E)]");
  DSV4_REQUIRE(block_size >= 1 && block_size <= 1024, "bad block_size %lld", (long long)block_size);
  DSV4_REQUIRE(num_tokens_post_pad && (m == 0 || (logits && topk_ids && topk_weights)) &&
                   (sorted_token_ids || sorted_capacity == 0) &&
                   (expert_ids || expert_ids_capacity == 0),
               "null pointer argument");
  const int64_t numel = m * topk;
  const int64_t need = align_capacity(numel, num_experts, block_size);
  DSV4_REQUIRE(sorted_capacity >= need, "sorted_token_ids capacity %lld < %lld",
               (long long)sorted_capacity, (long long)need);
  DSV4_REQUIRE(expert_ids_capacity * block_size >= need, "expert_ids capacity too small");
  const int64_t grid = router_align_grid(m);
  DSV4_REQUIRE(workspace != nullptr && workspace_words >= grid * num_experts,
               "workspace needs %lld int32 words", (long long)(grid * num_experts));
  const int epl = static_cast<int>((num_experts + 31) / 32);
  int m_i = static_cast<int>(m), e_i = static_cast<int>(num_experts), k_i = static_cast<int>(topk);
  int bm_i = static_cast<int>(block_size);
  int tpc = static_cast<int>((m + grid - 1) / grid);
  int cap_i = static_cast<int>(sorted_capacity), ecap_i = static_cast<int>(expert_ids_capacity);
  void* args[] = {&logits, &m_i, &e_i, &bias, &k_i, &renormalize, &scale, &bm_i, &tpc,
                  &topk_ids, &topk_weights, &sorted_token_ids, &cap_i, &expert_ids, &ecap_i,
                  &num_tokens_post_pad, &workspace, &slot_pos};
  const void* fn = router_align_fn(dtype, epl);
  if (fn == nullptr)
    return fail(DSV4_ERR_INVALID_ARGUMENT, "logits must be fp32, fp16, or bf16 (dtype %d)", dtype);
  cudaError_t e = cudaLaunchCooperativeKernel(fn, dim3(static_cast<unsigned>(grid)),
                                              dim3(kRouteAlignThreads), args,
                                              route_align_smem_bytes(e_i), as_stream(stream));
  if (e != cudaSuccess)
    return fail(DSV4_ERR_CUDA, "router_align_kernel: %s", cudaGetErrorString(e));
  return DSV4_OK;
}

int dsv4_b200_moe_align_block_size(const int32_t* topk_ids, int64_t numel, int64_t num_experts,
                                   int64_t block_size, int32_t* sorted_token_ids,
                                   int64_t sorted_capacity, int32_t* expert_ids,
                                   int64_t expert_ids_capacity, int32_t* num_tokens_post_pad,
                                   int32_t* cumsum_buffer, void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(num_experts >= 1 && num_experts <= kAlignMaxExperts,
               "num_experts must be in [1, %d], got %lld", kAlignMaxExperts,
               (long long)num_experts);
  DSV4_REQUIRE(block_size >= 1 && block_size <= 1024, "bad block_size %lld",
               (long long)block_size);
  DSV4_REQUIRE(numel >= 0 && numel < (1ll << 30), "bad numel %lld", (long long)numel);
  DSV4_REQUIRE(num_tokens_post_pad && (topk_ids || numel == 0) &&
                   (sorted_token_ids || sorted_capacity == 0) &&
                   (expert_ids || expert_ids_capacity == 0),
               "null pointer argument");
  const int64_t need = align_capacity(numel, num_experts, block_size);
  DSV4_REQUIRE(sorted_capacity >= need, "sorted_token_ids capacity %lld < %lld",
               (long long)sorted_capacity, (long long)need);
  DSV4_REQUIRE(expert_ids_capacity * block_size >= need, "expert_ids capacity too small");
  const int smem = align_smem_bytes(static_cast<int>(num_experts));
  launch_pdl(&moe_align_kernel, 1, kAlignThreads, smem, as_stream(stream), 
      topk_ids, static_cast<int>(numel), static_cast<int>(num_experts),
      static_cast<int>(block_size), sorted_token_ids, static_cast<int>(sorted_capacity),
      expert_ids, static_cast<int>(expert_ids_capacity), num_tokens_post_pad, cumsum_buffer,
      static_cast<int32_t*>(nullptr));
  return check_launch("moe_align_kernel");
}

int dsv4_b200_moe_align_workspace_words(int64_t numel, int64_t num_experts, int64_t* words) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(words != nullptr && numel >= 0 && num_experts >= 1, "bad arguments");
  *words = align_coop_grid(numel) * num_experts;
  return DSV4_OK;
}

int dsv4_b200_moe_align_block_size_ws(const int32_t* topk_ids, int64_t numel,
                                      int64_t num_experts, int64_t block_size,
                                      int32_t* sorted_token_ids, int64_t sorted_capacity,
                                      int32_t* expert_ids, int64_t expert_ids_capacity,
                                      int32_t* num_tokens_post_pad, int32_t* cumsum_buffer,
                                      int32_t* workspace, int64_t workspace_words,
                                      int32_t* slot_pos, void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(num_experts >= 1 && num_experts <= kAlignMaxExperts,
               "num_experts must be in [1, %d], got %lld", kAlignMaxExperts,
               (long long)num_experts);
  DSV4_REQUIRE(block_size >= 1 && block_size <= 1024, "bad block_size %lld",
               (long long)block_size);
  DSV4_REQUIRE(numel >= 0 && numel < (1ll << 30), "bad numel %lld", (long long)numel);
  DSV4_REQUIRE(num_tokens_post_pad && (topk_ids || numel == 0) &&
                   (sorted_token_ids || sorted_capacity == 0) &&
                   (expert_ids || expert_ids_capacity == 0),
               "null pointer argument");
  const int64_t need = align_capacity(numel, num_experts, block_size);
  DSV4_REQUIRE(sorted_capacity >= need, "sorted_token_ids capacity %lld < %lld",
               (long long)sorted_capacity, (long long)need);
  DSV4_REQUIRE(expert_ids_capacity * block_size >= need, "expert_ids capacity too small");
  const int64_t grid = align_coop_grid(numel);
  DSV4_REQUIRE(workspace != nullptr && workspace_words >= grid * num_experts,
               "workspace needs %lld int32 words", (long long)(grid * num_experts));
  int numel_i = static_cast<int>(numel), e_i = static_cast<int>(num_experts);
  int bm_i = static_cast<int>(block_size), ipc = static_cast<int>((numel + grid - 1) / grid);
  int cap_i = static_cast<int>(sorted_capacity), ecap_i = static_cast<int>(expert_ids_capacity);
  void* args[] = {&topk_ids, &numel_i, &e_i, &bm_i, &ipc, &sorted_token_ids, &cap_i,
                  &expert_ids, &ecap_i, &num_tokens_post_pad, &cumsum_buffer, &workspace,
                  &slot_pos};
  cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(&moe_align_coop_kernel),
                                              dim3(static_cast<unsigned>(grid)),
                                              dim3(kRouteAlignThreads), args,
                                              route_align_smem_bytes(e_i), as_stream(stream));
  if (e != cudaSuccess)
    return fail(DSV4_ERR_CUDA, "moe_align_coop_kernel: %s", cudaGetErrorString(e));
  return DSV4_OK;
}

int dsv4_b200_mxfp4_int8_moe_gemm(const int8_t* a_q, const float* a_scale, int64_t m_in,
                                  const uint8_t* b_mxfp4, const uint8_t* b_shift2,
                                  const float* b_channel_scale, int64_t num_experts, int64_t n,
                                  int64_t k, int64_t shift_stride, void* dst,
                                  const int32_t* sorted_token_ids, int64_t sorted_capacity,
                                  const int32_t* expert_ids, int64_t expert_ids_capacity,
                                  const int32_t* num_tokens_post_padded, int64_t topk,
                                  int64_t block_m, int source_rows_are_slots,
                                  int64_t num_valid_tokens, void* stream) {
  return moe_gemm_common(kEpiBf16, a_q, a_scale, m_in, b_mxfp4, b_shift2, b_channel_scale,
                         num_experts, n, k, shift_stride, dst, n, n / 128, 0, sorted_token_ids,
                         sorted_capacity, expert_ids, expert_ids_capacity, num_tokens_post_padded,
                         topk, block_m, source_rows_are_slots ? 1 : 0, num_valid_tokens, 0, 0.f,
                         stream);
}

int dsv4_b200_mxfp4_int8_moe_gemm_swiglu(
    const int8_t* a_q, const float* a_scale, int64_t m_in, const uint8_t* b_mxfp4,
    const uint8_t* b_shift2, const float* b_channel_scale, int64_t num_experts,
    int64_t intermediate, int64_t k, int64_t shift_stride, void* out,
    const int32_t* sorted_token_ids, int64_t sorted_capacity, const int32_t* expert_ids,
    int64_t expert_ids_capacity, const int32_t* num_tokens_post_padded, int64_t topk,
    int64_t block_m, int64_t num_valid_tokens, int has_clamp, float clamp_limit, void* stream) {
  DSV4_REQUIRE(intermediate > 0 && intermediate % 64 == 0,
               "intermediate_size must be a positive multiple of 64, got %lld",
               (long long)intermediate);
  return moe_gemm_common(kEpiSwiglu, a_q, a_scale, m_in, b_mxfp4, b_shift2, b_channel_scale,
                         num_experts, 2 * intermediate, k, shift_stride, out, intermediate,
                         intermediate / 64, intermediate, sorted_token_ids, sorted_capacity,
                         expert_ids, expert_ids_capacity, num_tokens_post_padded, topk, block_m,
                         0, num_valid_tokens, has_clamp, clamp_limit, stream);
}

// ---- expert-sorted row pipeline ----

int dsv4_b200_moe_sort_rows(const int8_t* a_q, const float* a_scale, int64_t m_in, int64_t k,
                            int64_t lda, int64_t scale_stride, const int32_t* sorted_token_ids, int64_t sorted_capacity,
                            const int32_t* num_tokens_post_padded, int64_t topk,
                            int source_rows_are_slots, int64_t num_valid_tokens, int8_t* out_q,
                            float* out_scale, int32_t* out_rowsum, void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(m_in >= 0 && k > 0 && k % 128 == 0, "K must be a positive multiple of 128");
  DSV4_REQUIRE(lda >= k && lda % 16 == 0 && scale_stride >= 1,
               "lda must be a multiple of 16 and >= K; scale_stride >= 1");
  DSV4_REQUIRE(topk >= 1 && topk <= 8, "topk must be in [1, 8], got %lld", (long long)topk);
  DSV4_REQUIRE(num_valid_tokens >= 0 && num_valid_tokens < (1ll << 31), "bad num_valid_tokens");
  if (sorted_capacity == 0 || m_in == 0) return DSV4_OK;
  DSV4_REQUIRE(a_q && a_scale && sorted_token_ids && num_tokens_post_padded && out_q && out_scale &&
                   out_rowsum,
               "null pointer argument");
  DSV4_REQUIRE((reinterpret_cast<uintptr_t>(a_q) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(out_q) & 15) == 0,
               "a_q and out_q must be 16-byte aligned");
  const int64_t blocks = (sorted_capacity + 7) / 8 < 4096 ? (sorted_capacity + 7) / 8 : 4096;
  launch_pdl(&sort_rows_kernel, static_cast<unsigned>(blocks), 256, 0, as_stream(stream), 
      a_q, a_scale, m_in, k, lda, scale_stride, sorted_token_ids, num_tokens_post_padded,
      sorted_capacity,
      static_cast<int>(topk), source_rows_are_slots ? 1 : 0, static_cast<int>(num_valid_tokens),
      out_q, out_scale, out_rowsum);
  return check_launch("sort_rows_kernel");
}

int dsv4_b200_quantize_sorted_int8(const void* a, int dtype, int64_t k,
                                   const int32_t* sorted_token_ids, int64_t sorted_capacity,
                                   const int32_t* num_tokens_post_padded,
                                   int64_t num_valid_tokens, int8_t* out_q, float* out_scale,
                                   int32_t* out_rowsum, void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(dtype == DSV4_BF16 || dtype == DSV4_F16, "a must be bf16 or fp16 (dtype %d)", dtype);
  DSV4_REQUIRE(k > 0 && k % 128 == 0 && k <= 8192, "K must be a multiple of 128 in [128, 8192]");
  DSV4_REQUIRE(num_valid_tokens >= 0 && num_valid_tokens < (1ll << 31), "bad num_valid_tokens");
  if (sorted_capacity == 0) return DSV4_OK;
  DSV4_REQUIRE(a && sorted_token_ids && num_tokens_post_padded && out_q && out_scale && out_rowsum,
               "null pointer argument");
  DSV4_REQUIRE((reinterpret_cast<uintptr_t>(a) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(out_q) & 7) == 0,
               "a must be 16-byte and out_q 8-byte aligned");
  cudaStream_t st = as_stream(stream);
  const bool wide = k > 2048;
  const int rows_per_cta = wide ? 2 : 8;
  const dim3 g(static_cast<unsigned>((sorted_capacity + rows_per_cta - 1) / rows_per_cta));
  const int nv = static_cast<int>(num_valid_tokens);
#define DSV4_QS(T, RT)                                                                        \
  launch_pdl(&quant_rows_reg_kernel<T, RT, 8>, g, 256, 0, st, static_cast<const T*>(a), sorted_capacity, \
                                                     k, k, 0.f, out_q, out_scale,               \
                                                     sorted_token_ids, num_tokens_post_padded,  \
                                                     nv, sorted_capacity, out_rowsum, 0)
  if (dtype == DSV4_BF16) {
    if (wide) DSV4_QS(__nv_bfloat16, 128); else DSV4_QS(__nv_bfloat16, 32);
  } else {
    if (wide) DSV4_QS(__half, 128); else DSV4_QS(__half, 32);
  }
#undef DSV4_QS
  return check_launch("quant_rows_reg_kernel (sorted)");
}

int dsv4_b200_quantize_sort_int8(const void* a, int dtype, int64_t m_in, int64_t k,
                                 const int32_t* sorted_token_ids, int64_t sorted_capacity,
                                 const int32_t* num_tokens_post_padded, int64_t topk,
                                 int64_t num_valid_tokens, int8_t* out_q, float* out_scale,
                                 int32_t* out_rowsum, void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(dtype == DSV4_BF16 || dtype == DSV4_F16, "a must be bf16 or fp16 (dtype %d)", dtype);
  DSV4_REQUIRE(k > 0 && k % 128 == 0 && k <= 8192, "K must be a multiple of 128 in [128, 8192]");
  DSV4_REQUIRE(topk >= 1 && topk <= 8, "topk must be in [1, 8], got %lld", (long long)topk);
  DSV4_REQUIRE(m_in >= 0 && num_valid_tokens >= 0 && num_valid_tokens <= m_in * topk &&
                   num_valid_tokens < (1ll << 31),
               "token rows do not cover num_valid_tokens");
  if (sorted_capacity == 0 || m_in == 0) return DSV4_OK;
  DSV4_REQUIRE(a && sorted_token_ids && num_tokens_post_padded && out_q && out_scale && out_rowsum,
               "null pointer argument");
  DSV4_REQUIRE((reinterpret_cast<uintptr_t>(a) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(out_q) & 7) == 0,
               "a must be 16-byte and out_q 8-byte aligned");
  cudaStream_t st = as_stream(stream);
  const bool wide = k > 2048;
  const int rows_per_cta = wide ? 2 : 8;
  const dim3 g(static_cast<unsigned>((sorted_capacity + rows_per_cta - 1) / rows_per_cta));
  const int nv = static_cast<int>(num_valid_tokens);
  const int tk = static_cast<int>(topk);
#define DSV4_QG(T, RT)                                                                          \
  launch_pdl(&quant_rows_reg_kernel<T, RT, 8>, g, 256, 0, st, static_cast<const T*>(a),          \
             sorted_capacity, k, k, 0.f, out_q, out_scale, sorted_token_ids,                     \
             num_tokens_post_padded, nv, sorted_capacity, out_rowsum, tk)
  if (dtype == DSV4_BF16) {
    if (wide) DSV4_QG(__nv_bfloat16, 128); else DSV4_QG(__nv_bfloat16, 32);
  } else {
    if (wide) DSV4_QG(__half, 128); else DSV4_QG(__half, 32);
  }
#undef DSV4_QG
  return check_launch("quant_rows_reg_kernel (quantise + sort)");
}

int dsv4_b200_quantize_scatter_int8(const void* a, int dtype, int64_t m_in, int64_t k,
                                    const int32_t* slot_pos, int64_t topk,
                                    int64_t num_valid_tokens, int64_t sorted_capacity,
                                    int8_t* out_q, float* out_scale, int32_t* out_rowsum,
                                    void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(dtype == DSV4_BF16 || dtype == DSV4_F16, "a must be bf16 or fp16 (dtype %d)", dtype);
  DSV4_REQUIRE(k > 0 && k % 128 == 0 && k <= 8192, "K must be a multiple of 128 in [128, 8192]");
  DSV4_REQUIRE(topk >= 1 && topk <= 32, "topk must be in [1, 32], got %lld", (long long)topk);
  DSV4_REQUIRE(m_in >= 0 && m_in < (1ll << 27) && num_valid_tokens >= 0 &&
                   num_valid_tokens <= m_in * topk,
               "token rows do not cover num_valid_tokens");
  DSV4_REQUIRE(sorted_capacity >= 0 && sorted_capacity < (1ll << 31), "bad sorted_capacity");
  if (sorted_capacity == 0 || m_in == 0 || num_valid_tokens == 0) return DSV4_OK;
  DSV4_REQUIRE(a && slot_pos && out_q && out_scale && out_rowsum, "null pointer argument");
  DSV4_REQUIRE((reinterpret_cast<uintptr_t>(a) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(out_q) & 7) == 0,
               "a must be 16-byte and out_q 8-byte aligned");
  cudaStream_t st = as_stream(stream);
  const bool wide = k > 2048;
  const int rows_per_cta = wide ? 2 : 8;
  const dim3 g(static_cast<unsigned>((m_in + rows_per_cta - 1) / rows_per_cta));
  const int nv = static_cast<int>(num_valid_tokens);
  const int tk = static_cast<int>(topk);
#define DSV4_QSC(T, RT)                                                                       \
  launch_pdl(&quant_scatter_kernel<T, RT, 8>, g, 256, 0, st, static_cast<const T*>(a), m_in, k, \
             k, slot_pos, tk, nv, sorted_capacity, out_q, out_scale, out_rowsum)
  if (dtype == DSV4_BF16) {
    if (wide) DSV4_QSC(__nv_bfloat16, 128); else DSV4_QSC(__nv_bfloat16, 32);
  } else {
    if (wide) DSV4_QSC(__half, 128); else DSV4_QSC(__half, 32);
  }
#undef DSV4_QSC
  return check_launch("quant_scatter_kernel");
}

int dsv4_b200_mxfp4_int8_moe_gemm_sorted(
    const int8_t* a_sorted, const float* a_scale, const int32_t* a_rowsum, const uint8_t* b_mxfp4, const uint8_t* b_shift2,
    const float* b_channel_scale, int64_t num_experts, int64_t n, int64_t k,
    int64_t shift_stride, void* dst, const int32_t* sorted_token_ids, int64_t sorted_capacity,
    const int32_t* expert_ids, int64_t expert_ids_capacity,
    const int32_t* num_tokens_post_padded, int64_t topk, int64_t block_m,
    int64_t num_valid_tokens, void* stream) {
  return moe_gemm_common(kEpiBf16, a_sorted, a_scale, sorted_capacity, b_mxfp4, b_shift2,
                         b_channel_scale, num_experts, n, k, shift_stride, dst, n, n / 128, 0,
                         sorted_token_ids, sorted_capacity, expert_ids, expert_ids_capacity,
                         num_tokens_post_padded, topk, block_m, 1, num_valid_tokens, 0, 0.f,
                         stream, true, a_rowsum);
}

int dsv4_b200_mxfp4_int8_moe_gemm_swiglu_sorted(
    const int8_t* a_sorted, const float* a_scale, const int32_t* a_rowsum, const uint8_t* b_mxfp4,
    const uint8_t* b_shift2, const float* b_channel_scale, int64_t num_experts,
    int64_t intermediate, int64_t k, int64_t shift_stride, void* out,
    const int32_t* sorted_token_ids, int64_t sorted_capacity, const int32_t* expert_ids,
    int64_t expert_ids_capacity, const int32_t* num_tokens_post_padded, int64_t topk,
    int64_t block_m, int64_t num_valid_tokens, int has_clamp, float clamp_limit, void* stream) {
  DSV4_REQUIRE(intermediate > 0 && intermediate % 64 == 0,
               "intermediate_size must be a positive multiple of 64, got %lld",
               (long long)intermediate);
  return moe_gemm_common(kEpiSwiglu, a_sorted, a_scale, sorted_capacity, b_mxfp4, b_shift2,
                         b_channel_scale, num_experts, 2 * intermediate, k, shift_stride, out,
                         intermediate, intermediate / 64, intermediate, sorted_token_ids,
                         sorted_capacity, expert_ids, expert_ids_capacity, num_tokens_post_padded,
                         topk, block_m, 0, num_valid_tokens, has_clamp, clamp_limit, stream, true,
                         a_rowsum);
}

int dsv4_b200_mxfp4_int8_moe_reduce(const void* routed_out, const float* topk_weights,
                                    void* out, int64_t m_out, int64_t n, int64_t topk,
                                    int64_t num_valid_tokens, int apply_scaling,
                                    float routed_scaling_factor, void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(n > 0 && n % 8 == 0, "reduce requires N divisible by 8, got %lld", (long long)n);
  DSV4_REQUIRE(topk >= 1 && topk <= 8, "topk must be in [1, 8], got %lld", (long long)topk);
  DSV4_REQUIRE(num_valid_tokens >= 0, "num_valid_tokens must be non-negative");
  DSV4_REQUIRE(m_out * topk >= num_valid_tokens, "out rows do not cover routed slots");
  if (m_out == 0) return DSV4_OK;
  DSV4_REQUIRE(routed_out && topk_weights && out, "null pointer argument");
  const int64_t threads = m_out * (n / 8);
  launch_pdl(&moe_reduce_kernel, static_cast<unsigned>((threads + 255) / 256), 256, 0, as_stream(stream), 
      static_cast<const __nv_bfloat16*>(routed_out), topk_weights,
      static_cast<__nv_bfloat16*>(out), static_cast<int>(m_out), static_cast<int>(n),
      static_cast<int>(topk), static_cast<int>(num_valid_tokens), routed_scaling_factor,
      apply_scaling ? 1 : 0);
  return check_launch("moe_reduce_kernel");
}

int dsv4_b200_mxfp4_int8_moe_reduce_masked(const void* routed_out, const float* topk_weights,
                                           const int32_t* topk_ids, void* out, int64_t m_out,
                                           int64_t n, int64_t topk, int64_t num_valid_tokens,
                                           int apply_scaling, float routed_scaling_factor,
                                           void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(n > 0 && n % 8 == 0, "reduce requires N divisible by 8, got %lld", (long long)n);
  DSV4_REQUIRE(topk >= 1 && topk <= 8, "topk must be in [1, 8], got %lld", (long long)topk);
  DSV4_REQUIRE(num_valid_tokens >= 0 && m_out * topk >= num_valid_tokens,
               "out rows do not cover routed slots");
  if (m_out == 0) return DSV4_OK;
  DSV4_REQUIRE(routed_out && topk_weights && topk_ids && out, "null pointer argument");
  const int64_t threads = m_out * (n / 8);
  launch_pdl(&moe_reduce_masked_kernel, static_cast<unsigned>((threads + 255) / 256), 256, 0,
                             as_stream(stream), 
      static_cast<const __nv_bfloat16*>(routed_out), topk_weights, topk_ids,
      static_cast<__nv_bfloat16*>(out), static_cast<int>(m_out), static_cast<int>(n),
      static_cast<int>(topk), static_cast<int>(num_valid_tokens), routed_scaling_factor,
      apply_scaling ? 1 : 0);
  return check_launch("moe_reduce_masked_kernel");
}

int dsv4_b200_gather_rows(const void* src, int64_t row_bytes, const int64_t* idx, int64_t n_rows,
                          void* dst, int64_t dst_stride, void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(row_bytes > 0 && row_bytes % 16 == 0, "row_bytes must be a multiple of 16");
  DSV4_REQUIRE(dst_stride >= row_bytes && dst_stride % 16 == 0,
               "dst_stride must be a multiple of 16 and >= row_bytes");
  DSV4_REQUIRE(n_rows >= 0, "bad n_rows");
  if (n_rows == 0) return DSV4_OK;
  DSV4_REQUIRE(idx && dst, "null pointer argument");
  DSV4_REQUIRE((reinterpret_cast<uintptr_t>(src) & 15) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0,
               "rows must be 16-byte aligned");
  const int64_t total = n_rows * (row_bytes / 16);
  const int64_t blocks = (total + 255) / 256 < 65535 ? (total + 255) / 256 : 65535;
  gather_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, as_stream(stream)>>>(
      static_cast<const uint8_t*>(src), row_bytes, idx, n_rows, static_cast<uint8_t*>(dst),
      dst_stride);
  return check_launch("gather_rows_kernel");
}

int dsv4_b200_ep_plan_fixed(const int32_t* topk_ids, const float* topk_weights,
                            const float* a_scale, int64_t m, int64_t topk, int64_t num_experts,
                            int64_t world, int64_t capacity, int64_t* send_src,
                            int32_t* send_meta, int64_t meta_words, int64_t meta_stride,
                            int64_t* pos, void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(world >= 1 && world <= 8 && num_experts % world == 0,
               "world must be in [1, 8] and divide num_experts");
  DSV4_REQUIRE(m >= 0 && m <= capacity && capacity < (1ll << 30), "need 0 <= m <= capacity");
  DSV4_REQUIRE(topk >= 1 && topk <= 8 && meta_words >= 1 + 2 * topk && meta_stride >= meta_words,
               "bad topk / meta width / meta stride");
  DSV4_REQUIRE(send_src && send_meta && (m == 0 || (topk_ids && topk_weights && a_scale && pos)),
               "null pointer argument");
  cudaStream_t st = as_stream(stream);
  ep_plan_fixed_kernel<<<1, kEpPlanThreads, 0, st>>>(
      topk_ids, static_cast<int>(m), static_cast<int>(topk), static_cast<int>(num_experts),
      static_cast<int>(world), static_cast<int>(capacity), send_src, pos);
  if (int r = check_launch("ep_plan_fixed_kernel")) return r;
  const int64_t words = world * capacity * meta_words;
  if (words == 0) return DSV4_OK;
  const int64_t blocks = (words + 255) / 256 < 4096 ? (words + 255) / 256 : 4096;
  ep_meta_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      topk_ids, topk_weights, a_scale, static_cast<int>(topk), static_cast<int>(num_experts),
      static_cast<int>(world), static_cast<int>(capacity), send_src, send_meta,
      static_cast<int>(meta_words), meta_stride);
  return check_launch("ep_meta_kernel");
}

int dsv4_b200_ep_combine(const void* partial, const int64_t* pos, int64_t world, void* out,
                         int64_t m, int64_t n, int apply_scaling, float routed_scaling_factor,
                         void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(n > 0 && n % 8 == 0, "combine requires N divisible by 8");
  DSV4_REQUIRE(world >= 1 && m >= 0, "bad world/m");
  if (m == 0) return DSV4_OK;
  DSV4_REQUIRE(pos && out, "null pointer argument");
  const int64_t threads = m * (n / 8);
  ep_combine_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16*>(partial), pos, static_cast<int>(world),
      static_cast<__nv_bfloat16*>(out), static_cast<int>(m), static_cast<int>(n),
      routed_scaling_factor, apply_scaling ? 1 : 0);
  return check_launch("ep_combine_kernel");
}

int dsv4_b200_mxfp4_int8_dense_gemm(const int8_t* a_q, const float* a_scale, int64_t m,
                                    int64_t k, const uint8_t* b_mxfp4, const uint8_t* b_shift2,
                                    int64_t shift_stride, const float* b_channel_scale, int64_t n,
                                    void* out, int32_t* partial, int64_t partial_splits,
                                    int64_t partial_ld, void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(m >= 0, "bad m");
  if (m == 0) return DSV4_OK;
  DSV4_REQUIRE(a_q && a_scale && b_mxfp4 && b_shift2 && b_channel_scale && out,
               "null pointer argument");
  DSV4_REQUIRE(m <= 0x7FFFFFFF, "m too large");
  const int64_t k_stages = (k / 32 + 7) / 8;  // 256-K stages of the GEMM kernel
  int64_t splits = 1;
  if (partial != nullptr && m <= 128 && partial_splits >= 2 && k_stages >= 2) {
    DSV4_REQUIRE(partial_ld >= n, "partial leading dimension %lld < N %lld",
                 (long long)partial_ld, (long long)n);
    const int64_t tiles = ((m + dense_tile(m) - 1) / dense_tile(m)) * (n / 128);
    splits = sm_count() / (tiles > 0 ? tiles : 1);
    if (splits < 2) splits = 2;
    if (splits > partial_splits) splits = partial_splits;
    if (splits > k_stages) splits = k_stages;
    const int64_t sps = (k_stages + splits - 1) / splits;
    splits = (k_stages + sps - 1) / sps;
  }
  if (splits > 1) {
    const int64_t split_stride = m * partial_ld;
    if (int r = dense_common(a_q, a_scale, m, k, b_mxfp4, b_shift2, shift_stride, b_channel_scale,
                             n, nullptr, partial, splits, partial_ld, split_stride, kEpiI32,
                             stream))
      return r;
    const int64_t total = m * n;
    launch_pdl(&splitk_reduce_kernel, static_cast<unsigned>((total + 255) / 256), 256, 0,
                           as_stream(stream), partial, static_cast<int>(splits), split_stride,
                                                partial_ld, a_scale, b_channel_scale,
                                                static_cast<__nv_bfloat16*>(out),
                                                static_cast<int>(m), static_cast<int>(n));
    return check_launch("splitk_reduce_kernel");
  }
  return dense_common(a_q, a_scale, m, k, b_mxfp4, b_shift2, shift_stride, b_channel_scale, n,
                      out, nullptr, 1, n, 0, kEpiBf16, stream);
}

int dsv4_b200_mxfp4_int8_dense_gemm_i32(const int8_t* a_q, int64_t m, int64_t k,
                                        const uint8_t* b_mxfp4, const uint8_t* b_shift2,
                                        int64_t shift_stride, int64_t n, int32_t* acc,
                                        void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(m >= 0, "bad m");
  if (m == 0) return DSV4_OK;
  DSV4_REQUIRE(a_q && b_mxfp4 && b_shift2 && acc, "null pointer argument");
  return dense_common(a_q, nullptr, m, k, b_mxfp4, b_shift2, shift_stride, nullptr, n, nullptr,
                      acc, 1, n, 0, kEpiI32, stream);
}

int dsv4_b200_quantize_per_token_int8_cm(const void* a, int dtype, int64_t m, int64_t k,
                                         int8_t* a_cm, float* a_scale, int32_t* a_rowsum,
                                         void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(dtype == DSV4_BF16 || dtype == DSV4_F16, "a must be bf16 or fp16 (dtype %d)", dtype);
  DSV4_REQUIRE(m >= 0 && m < (1ll << 31), "bad m");
  DSV4_REQUIRE(k > 0 && k % 128 == 0 && k <= 8192, "K must be a multiple of 128 in [128, 8192]");
  if (m == 0) return DSV4_OK;
  DSV4_REQUIRE(a && a_cm && a_scale && a_rowsum, "null pointer argument");
  DSV4_REQUIRE((reinterpret_cast<uintptr_t>(a) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(a_cm) & 7) == 0,
               "a must be 16-byte and a_cm 8-byte aligned");
  cudaStream_t st = as_stream(stream);
  const bool wide = k > 2048;
  const int rows_per_cta = wide ? 2 : 8;
  const dim3 g(static_cast<unsigned>((m + rows_per_cta - 1) / rows_per_cta));
#define DSV4_QC(T, RT)                                                                         \
  launch_pdl(&quant_rows_reg_kernel<T, RT, 8>, g, 256, 0, st, static_cast<const T*>(a), m, k, k, 0.f, a_cm, \
                                                     a_scale, nullptr, nullptr, 0, m, a_rowsum, 0)
  if (dtype == DSV4_BF16) {
    if (wide) DSV4_QC(__nv_bfloat16, 128); else DSV4_QC(__nv_bfloat16, 32);
  } else {
    if (wide) DSV4_QC(__half, 128); else DSV4_QC(__half, 32);
  }
#undef DSV4_QC
  return check_launch("quant_rows_reg_kernel (K-chunk-major)");
}

int dsv4_b200_rows_to_cm(const int8_t* a_q, int64_t m, int64_t k, int64_t lda, int8_t* a_cm,
                         int32_t* a_rowsum, void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(m >= 0 && m < (1ll << 31) && k > 0 && k % 128 == 0 && lda >= k && lda % 16 == 0,
               "bad shape m=%lld k=%lld lda=%lld", (long long)m, (long long)k, (long long)lda);
  if (m == 0) return DSV4_OK;
  DSV4_REQUIRE(a_q && a_cm && a_rowsum, "null pointer argument");
  DSV4_REQUIRE((reinterpret_cast<uintptr_t>(a_q) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(a_cm) & 15) == 0,
               "a_q and a_cm must be 16-byte aligned");
  const int64_t blocks = (m + 7) / 8 < 4096 ? (m + 7) / 8 : 4096;
  // identity permutation: a_scale is not copied (the caller's stays valid)
  launch_pdl(&sort_rows_kernel, static_cast<unsigned>(blocks), 256, 0, as_stream(stream), 
      a_q, nullptr, m, k, lda, 1, nullptr, nullptr, m, 1, 1, static_cast<int>(m), a_cm, nullptr,
      a_rowsum);
  return check_launch("sort_rows_kernel (identity)");
}

int dsv4_b200_mxfp4_int8_dense_gemm_cm(const int8_t* a_cm, const float* a_scale,
                                       const int32_t* a_rowsum, int64_t m, int64_t k,
                                       const uint8_t* b_mxfp4, const uint8_t* b_shift2,
                                       int64_t shift_stride, const float* b_channel_scale,
                                       int64_t n, void* out, void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(m >= 0 && m <= 0x7FFFFFFF, "bad m");
  if (m == 0) return DSV4_OK;
  DSV4_REQUIRE(a_cm && a_scale && a_rowsum && b_mxfp4 && b_shift2 && b_channel_scale && out,
               "null pointer argument");
  return dense_common(a_cm, a_scale, m, k, b_mxfp4, b_shift2, shift_stride, b_channel_scale, n,
                      out, nullptr, 1, n, 0, kEpiBf16, stream, a_rowsum);
}

// Allocation-free variant of dsv4_b200_mxfp4_int8_dense_gemm: the split-K
// workspace is the library's fixed device array (see the header for limits
// and the sharing rule).  Runs the same kernels as the allocating entry.
int dsv4_b200_mxfp4_int8_dense_gemm_noalloc(const int8_t* a_q, const float* a_scale, int64_t m,
                                            int64_t k, const uint8_t* b_mxfp4,
                                            const uint8_t* b_shift2, int64_t shift_stride,
                                            const float* b_channel_scale, int64_t n, void* out,
                                            void* stream) {
  if (int r = ensure_init()) return r;
  DSV4_REQUIRE(m >= 0 && n > 0, "bad shape m=%lld n=%lld", (long long)m, (long long)n);
  const int64_t ld = (n + 31) / 32 * 32;
  const int64_t splits = 4;
  DSV4_REQUIRE(m <= 128 && splits * m * ld <= kNoAllocScratchWords,
               "dense_gemm_noalloc: m=%lld, n=%lld exceed the fixed split-K workspace "
               "(m <= 128 and 4*m*ceil32(n) <= %lld int32 words)",
               (long long)m, (long long)n, (long long)kNoAllocScratchWords);
  int32_t* scratch = nullptr;
  if (int r = noalloc_scratch(&scratch)) return r;
  return dsv4_b200_mxfp4_int8_dense_gemm(a_q, a_scale, m, k, b_mxfp4, b_shift2, shift_stride,
                                         b_channel_scale, n, out, scratch, splits, ld, stream);
}

#ifdef DSV4_TRACE
DSV4_API int dsv4_b200_debug_trace(long long* host, int reset) {
  cudaMemcpyFromSymbol(host, g_trace, sizeof(g_trace));
  if (reset) {
    static long long zeros[kTraceEvents][kTraceStages];
    cudaMemcpyToSymbol(g_trace, zeros, sizeof(g_trace));
  }
  return DSV4_OK;
}
#endif

}  // extern "C"
