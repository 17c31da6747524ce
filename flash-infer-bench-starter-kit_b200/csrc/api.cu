// C ABI and host orchestration of the fused FP8 DeepSeek-V3 MoE layer.
//
// Replaces the host pipeline run(...) of the reference
// (solution/python/main.cpp:66-266): the same six steps (route, count/scan,
// permute+gather, GEMM1+SwiGLU, GEMM2, combine) as six kernel launches on the
// caller's stream, with every intermediate carved out of one caller-owned
// workspace instead of ~25 per-call torch allocations, and no host sync.
#include <mutex>
#include <string.h>

#include "kernels.cuh"

namespace moe {
namespace {

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  bool init = false;
  int sm_count = 0;
  int major = 0;
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_mu;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
int g_bn_override[2] = {0, 0};
int g_path_override = 0;          // 0 automatic, 1 weights-on-M e4m3 GEMMs, 2 tokens-on-M e4m3 GEMMs
// From this batch size the layer runs the tokens-on-M e4m3 GEMMs (gemm_tm.cu).
constexpr int kTmMinTokens = 1280;
cudaEvent_t g_stage_events[7] = {};
bool g_stage_events_on = false;

// The CUDA error behind the calling thread's last MOE_ERR_CUDA.
thread_local cudaError_t g_last_cuda_error = cudaSuccess;

int cuda_fail(cudaError_t e) {
  g_last_cuda_error = e;
  return MOE_ERR_CUDA;
}

void mark_stage(int i, cudaStream_t s) {
  if (g_stage_events_on) cudaEventRecord(g_stage_events[i], s);
}

int device_info(DeviceInfo* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MOE_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.init) {
    if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return MOE_ERR_NO_DEVICE;
    if (cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return MOE_ERR_NO_DEVICE;
    d.init = true;
  }
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return MOE_ERR_NO_DEVICE;
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  *out = d;
  return d.major == 10 ? MOE_OK : MOE_ERR_NO_DEVICE;
}

}  // namespace

void* current_cu_context() {
  using CtxGetCurrentFn = CUresult (*)(CUcontext*);
  static std::atomic<CtxGetCurrentFn> fn_cache{nullptr};
  CtxGetCurrentFn fn = fn_cache.load(std::memory_order_acquire);
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !p)
      return nullptr;
    fn = reinterpret_cast<CtxGetCurrentFn>(p);
    fn_cache.store(fn, std::memory_order_release);
  }
  CUcontext ctx = nullptr;
  return fn(&ctx) == CUDA_SUCCESS ? static_cast<void*>(ctx) : nullptr;
}

namespace {

// Token-tile widths of the weights-on-M GEMM1 and GEMM2 from the expected
// tokens per active expert (T*8/256).  Measured on B200 with 32 local experts
// (layer us, GEMM1/GEMM2 widths): T=64 16/16 155 vs 16/32 159; T=128 191 vs
// 184; T=384 277 vs 269; T=512 32/32 297 vs 16/32 305 and 64/64 328; T=640
// 64/64 324 vs 32/32 334; T=768 353 vs 367; T=1024 64/64 387 vs 32/32 422.
void pick_bn(int T, int E_l, int* bn1, int* bn2) {
  const double per_expert = (double)T * kTopK / kExpertsGlobal;
  (void)E_l;
  if (per_expert <= 2.0) { *bn1 = 16; *bn2 = 16; }
  else if (per_expert <= 12.0) { *bn1 = 16; *bn2 = 32; }
  else if (per_expert <= 16.0) { *bn1 = 32; *bn2 = 32; }
  else if (per_expert <= 48.0) { *bn1 = 64; *bn2 = 64; }
  else { *bn1 = 64; *bn2 = 128; }
}

struct Plan {
  moe_fp8_ds_layout pub;
  int T, E_l, NB, NB8, R_cap, bn1, bn2, grid1, grid2, max_mt1, max_mt2;
  bool tm;                          // large batch: tokens-on-M e4m3 GEMMs (gemm_tm.cu)
  uint64_t tiles1, tiles2, sched, counters1, counters2, ready, partials1, partials2, front_sync;
};

uint64_t align256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

void make_plan(int T, int E_l, int sm_count, Plan* P) {
  memset(P, 0, sizeof(*P));
  // The tuning knobs may be changed by another thread: one snapshot per plan.
  int bn_override[2], path_override;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    bn_override[0] = g_bn_override[0];
    bn_override[1] = g_bn_override[1];
    path_override = g_path_override;
  }
  P->T = T;
  P->E_l = E_l;
  P->NB = (T + kPermBlock - 1) / kPermBlock;
  // row capacity, a multiple of 16 so that per-row fp32 arrays [blocks][R_cap]
  // have 16-byte-aligned rows (TMA boxes of the tokens-on-M GEMMs)
  P->R_cap = (T * (E_l < kTopK ? E_l : kTopK) + 15) & ~15;
  // GEMM1 keeps X1 and X2 accumulators of 128 features per token column in
  // registers, so its widest tile is 64 tokens (128 would need the whole
  // register file); GEMM2 holds one accumulator and goes to 128.
  int bn_auto1 = 16, bn_auto2 = 16;
  pick_bn(T, E_l, &bn_auto1, &bn_auto2);
  // Tokens-on-M GEMMs (gemm_tm.cu) from kTmMinTokens: their 128-row token
  // tiles fill the MMA once experts see ~40+ tokens each.  Below that the
  // weights-on-M GEMMs (gemm_fp8.cu) size the MMA's N to the few tokens an
  // expert has.  Measured on B200 with 32 local experts, layer us
  // weights-on-M / tokens-on-M: T=1024 387/411, 1280 448/443, 1536 487/451,
  // 2048 575/455, 4096 932/664, 8192 1697/1108.
  P->tm = path_override == 2 || (path_override == 0 && T >= kTmMinTokens);
  if (P->tm) {
    // One token tile holds up to 128 rows of one expert (the MMA's M side); a
    // smaller tile cap may be forced for tests.
    auto cap = [](int v) { return v > 0 && v <= 128 ? v : 128; };
    P->bn1 = P->bn2 = cap(bn_override[0]);
  } else {
    // e4m3 kernels are compiled for 16, 32, 64 and 128 tokens only.
    auto compiled = [](int v) { return v == 16 || v == 32 || v == 64 || v == 128; };
    P->bn1 = compiled(bn_override[0]) ? bn_override[0] : bn_auto1;
    P->bn2 = compiled(bn_override[1]) ? bn_override[1] : bn_auto2;
  }

  auto max_mt = [&](int bn) {
    long v = (long)P->R_cap / bn + E_l;
    return (int)(v < P->R_cap ? v : P->R_cap);
  };
  P->max_mt1 = max_mt(P->bn1);
  P->max_mt2 = max_mt(P->bn2);
  uint64_t off = 0;
  auto take = [&](uint64_t bytes) { uint64_t o = off; off = align256(off + bytes); return o; };
  const uint64_t R = (uint64_t)P->R_cap;
  P->pub.error_word = take(16);
  P->pub.topk_ids = take((uint64_t)T * kTopK * 4);
  P->pub.topk_weights = take((uint64_t)T * kTopK * 4);
  P->pub.inv_row = take((uint64_t)T * kTopK * 4);
  P->NB8 = 4 * P->NB;                     // byte-mask row length, padded to whole 32-token blocks
  P->pub.block_masks = take((uint64_t)P->NB8 * E_l);
  P->pub.block_bases = take((uint64_t)P->NB * E_l * 4);
  P->pub.seg_offsets = take((uint64_t)(E_l + 1) * 4);
  P->tiles1 = take((uint64_t)P->max_mt1 * 16);
  P->tiles2 = take((uint64_t)P->max_mt2 * 16);
  P->sched = take(64);
  P->front_sync = take(16);
  P->counters1 = take((uint64_t)P->max_mt1 * (kInter / 128) * 4);
  P->counters2 = take((uint64_t)P->max_mt2 * (kHidden / 128) * 4);
  P->ready = take((uint64_t)E_l * 4);
  P->pub.row_token = take(R * 4);
  // (the tokens-on-M GEMMs' intermediate holds the hi and lo planes
  // [2][R_cap][2048] in the same bytes as the weights-on-M row pairs)
  P->pub.act = take(R * kHidden);
  P->pub.act_scale = take(R * kHiddenBlocks * 4);
  P->pub.inter = take(2 * R * kInter);
  P->pub.inter_scale = take(R * kInterBlocks * 4);
  P->pub.down = take(R * kHidden * 4);
  if (P->tm) {
    P->grid1 = P->grid2 = sm_count;
    P->partials1 = take(gemm_tm_partials_bytes(P->grid1));
    P->partials2 = take(gemm_tm_partials_bytes(P->grid2));
  } else {
    P->grid1 = sm_count * gemm_ctas_per_sm(1, P->bn1);   // persistent: every resident CTA slot
    P->grid2 = sm_count * gemm_ctas_per_sm(2, P->bn2);
    P->partials1 = take(gemm_partials_bytes(1, P->bn1, P->grid1));
    P->partials2 = take(gemm_partials_bytes(2, P->bn2, P->grid2));
  }
  P->pub.total_bytes = off;
  P->pub.row_capacity = P->R_cap;
}

// 3D view of a K-major e4m3 matrix [rows, K]: x = byte inside a 128-wide K
// block, y = row, z = K block; a box covers box_rows rows x kblocks K blocks,
// landing as kblocks consecutive 128-byte-swizzled [box_rows x 128] tiles.
// 2D view of a K-major e4m3 matrix [rows, K] with a 128-byte x 1-row box, for
// tile::gather4 row gathers.
bool encode_rows_2d(CUtensorMap* m, const void* base, uint64_t K, uint64_t rows) {
  cuuint64_t dims[2] = {K, rows};
  cuuint64_t strides[1] = {K};
  cuuint32_t box[2] = {128, 1};
  cuuint32_t estr[2] = {1, 1};
  return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_kmajor(CUtensorMap* m, const void* base, uint64_t K, uint64_t rows, uint32_t box_rows,
                   uint32_t kblocks) {
  cuuint64_t dims[3] = {128, rows, K / 128};
  cuuint64_t strides[2] = {K, 128};         // bytes (1-byte elements)
  cuuint32_t box[3] = {128, box_rows, kblocks};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// K-major e4m3 operand in two planes, viewed as {128 B of a K block, row, K
// block, plane}: W13 [E_l][2][2048][7168] (plane = expert*2 + X1|X2) or the
// intermediate [2][R_cap][2048] (plane = hi|lo).  A box covers box_rows rows
// x kblocks K blocks x 2 planes, landing as [plane][K block][row][128 B]
// with 128-byte swizzling.
bool encode_kmajor_planes(CUtensorMap* m, const void* base, uint64_t K, uint64_t rows, uint64_t planes,
                          uint32_t box_rows, uint32_t kblocks) {
  cuuint64_t dims[4] = {128, rows, K / 128, planes};
  cuuint64_t strides[3] = {K, 128, rows * K};
  cuuint32_t box[4] = {128, box_rows, kblocks, 2};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// fp32 [rows][cols] row-major (cols * 4 a multiple of 16 bytes); box = box_cols x box_rows.
bool encode_f32_2d(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint32_t box_cols,
                   uint32_t box_rows) {
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 4};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// fp32 [d2][d1][d0] row-major; box = b0 x b1 x b2.
bool encode_f32_3d(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint32_t b0,
                   uint32_t b1, uint32_t b2) {
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * 4, d0 * d1 * 4};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int validate_common(const moe_fp8_ds_args* a, bool routed) {
  if (!a) return MOE_ERR_INVALID_ARGUMENT;
  if (a->num_tokens < 0 || a->num_local_experts < 1 || a->num_local_experts > kExpertsGlobal)
    return MOE_ERR_INVALID_ARGUMENT;
  if (a->num_tokens > (1 << 20)) return MOE_ERR_TOO_LARGE;
  if (a->num_tokens == 0) return MOE_OK;
  const void* need[] = {a->hidden_states, a->hidden_states_scale, a->gemm1_weights,
                        a->gemm1_weights_scale, a->gemm2_weights, a->gemm2_weights_scale};
  for (const void* p : need) if (!p) return MOE_ERR_INVALID_ARGUMENT;
  if (!a->output && !a->output_f32) return MOE_ERR_INVALID_ARGUMENT;
  if (routed) {
    if (!a->topk_ids || !a->topk_weights) return MOE_ERR_INVALID_ARGUMENT;
  } else {
    if (!a->routing_logits || !a->routing_bias) return MOE_ERR_INVALID_ARGUMENT;
    if (!aligned16(a->routing_logits) || !aligned16(a->routing_bias)) return MOE_ERR_MISALIGNED;
  }
  if (!aligned16(a->hidden_states) || !aligned16(a->gemm1_weights) || !aligned16(a->gemm2_weights) ||
      !aligned16(a->output ? a->output : a->output_f32))
    return MOE_ERR_MISALIGNED;
  return MOE_OK;
}

int run_impl(const moe_fp8_ds_args* a, void* ws, uint64_t ws_bytes, void* stream, bool routed) {
  int st = validate_common(a, routed);
  if (st != MOE_OK) return st;
  const int T = a->num_tokens, E_l = a->num_local_experts;
  if (T == 0) return MOE_OK;
  DeviceInfo dev;
  st = device_info(&dev);
  if (st != MOE_OK) return st;
  Plan P;
  make_plan(T, E_l, dev.sm_count, &P);
  if (!ws || (reinterpret_cast<uintptr_t>(ws) & 255)) return MOE_ERR_MISALIGNED;
  if (ws_bytes < P.pub.total_bytes) return MOE_ERR_WORKSPACE_TOO_SMALL;
  uint8_t* base = static_cast<uint8_t*>(ws);
  auto at = [&](uint64_t off) { return base + off; };
  int* err = reinterpret_cast<int*>(at(P.pub.error_word));
  int32_t* ids = routed ? const_cast<int32_t*>(a->topk_ids) : reinterpret_cast<int32_t*>(at(P.pub.topk_ids));
  float* wts = routed ? const_cast<float*>(a->topk_weights) : reinterpret_cast<float*>(at(P.pub.topk_weights));
  int32_t* inv = reinterpret_cast<int32_t*>(at(P.pub.inv_row));
  uint8_t* masks8 = at(P.pub.block_masks);
  uint8_t* act = at(P.pub.act);
  float* act_scale = reinterpret_cast<float*>(at(P.pub.act_scale));
  int32_t* bases = reinterpret_cast<int32_t*>(at(P.pub.block_bases));
  int32_t* seg = reinterpret_cast<int32_t*>(at(P.pub.seg_offsets));
  int4* tiles1 = reinterpret_cast<int4*>(at(P.tiles1));
  int4* tiles2 = reinterpret_cast<int4*>(at(P.tiles2));
  int32_t* sched = reinterpret_cast<int32_t*>(at(P.sched));
  int32_t* cnt1 = reinterpret_cast<int32_t*>(at(P.counters1));
  int32_t* cnt2 = reinterpret_cast<int32_t*>(at(P.counters2));
  int* ready = reinterpret_cast<int*>(at(P.ready));
  int32_t* row_token = reinterpret_cast<int32_t*>(at(P.pub.row_token));
  uint8_t* inter = at(P.pub.inter);
  float* inter_scale = reinterpret_cast<float*>(at(P.pub.inter_scale));
  float* down = reinterpret_cast<float*>(at(P.pub.down));
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  CUtensorMap tm_w1, tm_b1, tm_w2, tm_b2;
  CUtensorMap tm_bs1, tm_ws1, tm_bs2, tm_ws2;   // tokens-on-M GEMMs: block scales
  if (P.tm) {
    // tokens-on-M GEMMs: 128-row boxes of tokens (GEMM2: hi plane rows r, lo
    // plane rows R_cap + r) and of weights
    const uint32_t ks1 = (uint32_t)gemm_tm_k_per_stage(1), ks2 = (uint32_t)gemm_tm_k_per_stage(2);
    if (!encode_kmajor_planes(&tm_w1, a->gemm1_weights, kHidden, kInter, 2ull * E_l, 128, ks1) ||
        !encode_kmajor(&tm_b1, act, kHidden, (uint64_t)P.R_cap, 128, ks1) ||
        !encode_kmajor(&tm_w2, a->gemm2_weights, kInter, (uint64_t)E_l * kHidden, 128, ks2) ||
        !encode_kmajor_planes(&tm_b2, inter, kInter, (uint64_t)P.R_cap, 2, 128, ks2))
      return MOE_ERR_INVALID_ARGUMENT;
    // token scales [K blocks][R_cap]: boxes of 132 rows x the stage's K blocks;
    // weight scales: 4 K blocks of each half's 128-row block
    const uint32_t sbox = (uint32_t)gemm_tm_scale_box_cols();
    if (!aligned16(a->gemm1_weights_scale) || !aligned16(a->gemm2_weights_scale))
      return MOE_ERR_MISALIGNED;
    if (!encode_f32_2d(&tm_bs1, act_scale, (uint64_t)P.R_cap, kHiddenBlocks, sbox, ks1) ||
        !encode_f32_2d(&tm_bs2, inter_scale, (uint64_t)P.R_cap, kInterBlocks, sbox, ks2) ||
        !encode_f32_3d(&tm_ws1, a->gemm1_weights_scale, kHiddenBlocks, kInter / 128, 2ull * E_l, 4, 1, 2) ||
        !encode_f32_3d(&tm_ws2, a->gemm2_weights_scale, kInterBlocks, kHidden / 128, (uint64_t)E_l, 4, 1, 1))
      return MOE_ERR_INVALID_ARGUMENT;
  } else {
  const uint32_t ks1 = (uint32_t)gemm_k_per_stage(1, P.bn1), ks2 = (uint32_t)gemm_k_per_stage(2, P.bn2);
  // After the fused front kernel (T <= 256, 16-token tiles) GEMM1 gathers token
  // rows itself: a map of hidden_states with 128-byte x 1-row boxes
  // (tile::gather4), rows by row_token.  With wider tiles (larger T) the four
  // rows per copy cost more than the scatter kernel's copy: measured T=1024
  // 422 vs 387 us, so there the permuted activation is materialised.
  const bool gather1 = !routed && T <= kFrontMaxTokens && P.bn1 <= kGatherMaxBN;
  if (!encode_kmajor(&tm_w1, a->gemm1_weights, kHidden, (uint64_t)E_l * kGemm1Out, 128, ks1) ||
      !(gather1 ? encode_rows_2d(&tm_b1, a->hidden_states, kHidden, (uint64_t)T)
                : encode_kmajor(&tm_b1, act, kHidden, (uint64_t)P.R_cap, (uint32_t)P.bn1, ks1)) ||
      !encode_kmajor(&tm_w2, a->gemm2_weights, kInter, (uint64_t)E_l * kHidden, 128, ks2) ||
      !encode_kmajor(&tm_b2, inter, kInter, 2ull * P.R_cap, (uint32_t)(2 * P.bn2), ks2))
    return MOE_ERR_INVALID_ARGUMENT;
  }

  cudaError_t ce;
  const bool front = !routed && T <= kFrontMaxTokens && !P.tm && P.bn1 <= kGatherMaxBN;
  if (front) {
    // Small batch: routing, row assignment and gather in one launch.
    mark_stage(0, s);
    ce = launch_front(a->routing_logits, a->routing_bias, T, a->routed_scaling_factor,
                      a->local_expert_offset, E_l, P.R_cap, P.bn1, P.bn2, kInter / 128, kHidden / 128,
                      a->hidden_states, a->hidden_states_scale, ids, wts, masks8, P.NB8, seg, tiles1, tiles2,
                      sched, cnt1, cnt2, ready, inv, row_token, act, act_scale, err,
                      reinterpret_cast<int*>(at(P.front_sync)), s);
    if (ce != cudaSuccess) return cuda_fail(ce);
    mark_stage(1, s);
    mark_stage(2, s);
  } else {
    mark_stage(0, s);
    ce = launch_route(routed, a->routing_logits, a->routing_bias, T, a->routed_scaling_factor,
                      a->local_expert_offset, E_l, ids, wts, masks8, P.NB8, err, s);
    if (ce != cudaSuccess) return cuda_fail(ce);
    mark_stage(1, s);
    ce = launch_scan(masks8, P.NB8, bases, P.NB, E_l, seg, P.bn1, P.bn2, tiles1, tiles2, sched, cnt1,
                     P.tm ? gemm_tm_units_per_tile(1) : kInter / 128, cnt2,
                     P.tm ? gemm_tm_units_per_tile(2) : kHidden / 128, ready, s);
    if (ce != cudaSuccess) return cuda_fail(ce);
    mark_stage(2, s);
    ce = launch_scatter(ids, masks8, P.NB8, bases, T, E_l, a->local_expert_offset, P.R_cap,
                        a->hidden_states, a->hidden_states_scale, inv, row_token, act, act_scale, s);
    if (ce != cudaSuccess) return cuda_fail(ce);
  }

  GemmParams g1{};
  g1.tiles = tiles1; g1.sched = sched; g1.w_scale = a->gemm1_weights_scale;
  g1.b_scale = act_scale;
  g1.counters = cnt1; g1.ready = ready; g1.bn_prev = 0;
  g1.early_start = front ? 1 : 0; g1.partials = reinterpret_cast<float*>(at(P.partials1));
  g1.inter = inter; g1.inter_scale = inter_scale; g1.down = nullptr; g1.err = err; g1.R_cap = P.R_cap;
  mark_stage(3, s);
  g1.front_sync = front ? reinterpret_cast<int*>(at(P.front_sync)) : nullptr;
  g1.row_token = front ? row_token : nullptr;   // GEMM1 gathers token rows by row_token
  g1.front_ctas = (T + kRouteTokens - 1) / kRouteTokens;
  ce = P.tm     ? launch_gemm_tm(1, &tm_w1, &tm_b1, &tm_bs1, &tm_ws1, g1, P.grid1, s)
                : launch_gemm(1, P.bn1, &tm_w1, &tm_b1, g1, P.grid1, s);
  if (ce != cudaSuccess) return cuda_fail(ce);

  GemmParams g2{};
  g2.tiles = tiles2; g2.sched = sched; g2.w_scale = a->gemm2_weights_scale;
  g2.b_scale = inter_scale;
  g2.counters = cnt2; g2.ready = ready; g2.seg = seg; g2.bn_prev = P.bn1;
  g2.early_start = front ? 1 : 0; g2.partials = reinterpret_cast<float*>(at(P.partials2));
  g2.inter = nullptr; g2.inter_scale = nullptr; g2.down = down; g2.err = err; g2.R_cap = P.R_cap;
  mark_stage(4, s);
  ce = P.tm     ? launch_gemm_tm(2, &tm_w2, &tm_b2, &tm_bs2, &tm_ws2, g2, P.grid2, s)
                : launch_gemm(2, P.bn2, &tm_w2, &tm_b2, g2, P.grid2, s);
  if (ce != cudaSuccess) return cuda_fail(ce);

  mark_stage(5, s);
  ce = launch_combine(down, inv, wts, T, a->output, a->output_f32,
                      front ? reinterpret_cast<int*>(at(P.front_sync)) : nullptr, err, s);
  if (ce != cudaSuccess) return cuda_fail(ce);
  mark_stage(6, s);
  return MOE_OK;
}

}  // namespace

// Internal entry for other translation units of this library.
int run_layer_with_workspace(const moe_fp8_ds_args* a, void* ws, uint64_t ws_bytes, void* stream,
                             bool routed) {
  return run_impl(a, ws, ws_bytes, stream, routed);
}

}  // namespace moe

using namespace moe;

namespace moe {
// Failure-detection self test: one thread waits, with the bounded wait every
// pipeline wait uses, on a counter nothing increments (word 3 of the
// workspace's error block, zeroed by the host first).  When the wait gives up
// it records kDevTimeoutBarrier in the error word and the kernel returns, so
// the context stays usable.
__global__ void selftest_wait_kernel(int* words) {
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    if (!wait_counter(words + 3, 1, &abort_flag)) raise_error(words, kDevTimeoutBarrier);
  }
}
}  // namespace moe

extern "C" {

int moe_fp8_ds_workspace_layout(int32_t num_tokens, int32_t num_local_experts,
                                moe_fp8_ds_layout* layout) {
  if (!layout || num_tokens < 0 || num_local_experts < 1 || num_local_experts > kExpertsGlobal)
    return MOE_ERR_INVALID_ARGUMENT;
  if (num_tokens > (1 << 20)) return MOE_ERR_TOO_LARGE;
  DeviceInfo dev;
  int st = device_info(&dev);
  if (st != MOE_OK) return st;
  Plan P;
  make_plan(num_tokens, num_local_experts, dev.sm_count, &P);
  *layout = P.pub;
  return MOE_OK;
}

int moe_fp8_ds_workspace_size(int32_t num_tokens, int32_t num_local_experts, uint64_t* bytes) {
  if (!bytes) return MOE_ERR_INVALID_ARGUMENT;
  moe_fp8_ds_layout l;
  int st = moe_fp8_ds_workspace_layout(num_tokens, num_local_experts, &l);
  if (st != MOE_OK) return st;
  *bytes = l.total_bytes;
  return MOE_OK;
}

int moe_fp8_ds_run(const moe_fp8_ds_args* args, void* workspace, uint64_t workspace_bytes,
                   void* stream) {
  return run_impl(args, workspace, workspace_bytes, stream, false);
}

int moe_fp8_ds_run_routed(const moe_fp8_ds_args* args, void* workspace, uint64_t workspace_bytes,
                          void* stream) {
  return run_impl(args, workspace, workspace_bytes, stream, true);
}

int moe_fp8_ds_route(const float* routing_logits, const void* routing_bias, int32_t num_tokens,
                     float routed_scaling_factor, int32_t* topk_ids, float* topk_weights,
                     void* stream) {
  if (num_tokens < 0 || (num_tokens > 0 && (!routing_logits || !routing_bias || !topk_ids || !topk_weights)))
    return MOE_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return MOE_OK;
  DeviceInfo dev;
  int st = device_info(&dev);
  if (st != MOE_OK) return st;
  // No local experts (E_l = 0, no histogram): routing only.
  cudaError_t ce = launch_route(false, routing_logits, routing_bias, num_tokens,
                                routed_scaling_factor, 0, 0, topk_ids, topk_weights, nullptr, 0,
                                nullptr, static_cast<cudaStream_t>(stream));
  return ce == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

int moe_fp8_ds_selftest_wait_timeout(void* workspace, void* stream) {
  if (!workspace) return MOE_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return MOE_ERR_MISALIGNED;
  DeviceInfo di;
  const int st = device_info(&di);
  if (st != MOE_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* words = static_cast<int*>(workspace);
  if (cudaMemsetAsync(words + 3, 0, 4, s) != cudaSuccess) return MOE_ERR_CUDA;
  moe::selftest_wait_kernel<<<1, 32, 0, s>>>(words);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

int moe_fp8_ds_read_device_error(void* workspace, void* stream, int32_t* device_error) {
  if (!workspace || !device_error) return MOE_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t v = 0;
  if (cudaMemcpyAsync(&v, workspace, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess) return MOE_ERR_CUDA;
  if (cudaMemsetAsync(workspace, 0, 16, s) != cudaSuccess) return MOE_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return MOE_ERR_CUDA;
  *device_error = v;
  if (v == kDevOk) return MOE_OK;
  if (v == kDevTimeoutProducer || v == kDevTimeoutMma || v == kDevTimeoutEpilogue ||
      v == kDevTimeoutBarrier)
    return MOE_ERR_DEVICE_TIMEOUT;
  return MOE_ERR_DEVICE_FAULT;
}

const char* moe_fp8_ds_last_cuda_error_string(void) {
  return cudaGetErrorString(g_last_cuda_error);
}

const char* moe_fp8_ds_status_string(int status) {
  switch (status) {
    case MOE_OK: return "ok";
    case MOE_ERR_INVALID_ARGUMENT: return "invalid argument";
    case MOE_ERR_MISALIGNED: return "pointer not 16-byte aligned (workspace: 256-byte)";
    case MOE_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case MOE_ERR_CUDA: return "CUDA runtime error";
    case MOE_ERR_NO_DEVICE: return "no sm_100 device or driver entry point";
    case MOE_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case MOE_ERR_DEVICE_FAULT: return "device-side check failed";
    case MOE_ERR_TOO_LARGE: return "size exceeds the entry point's limit";
  }
  return "unknown status";
}

int moe_fp8_ds_set_tile_override(int32_t bn_gemm1, int32_t bn_gemm2) {
  auto ok = [](int v) { return v >= 0 && v <= 256 && v % 16 == 0; };
  if (!ok(bn_gemm1) || !ok(bn_gemm2)) return MOE_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lk(g_mu);
  g_bn_override[0] = bn_gemm1;
  g_bn_override[1] = bn_gemm2;
  return MOE_OK;
}

int moe_fp8_ds_set_stage_events(void* const* events, int32_t count) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (count == 0) { g_stage_events_on = false; return MOE_OK; }
  if (count != 7 || !events) return MOE_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < 7; ++i) {
    if (!events[i]) return MOE_ERR_INVALID_ARGUMENT;
    g_stage_events[i] = static_cast<cudaEvent_t>(events[i]);
  }
  g_stage_events_on = true;
  return MOE_OK;
}

int moe_fp8_ds_set_path_override(int32_t mode) {
  if (mode < 0 || mode > 2) return MOE_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lk(g_mu);
  g_path_override = mode;
  return MOE_OK;
}

int moe_fp8_ds_launches_per_call(int32_t num_tokens) {
  if (num_tokens <= 0) return 0;
  return num_tokens <= kFrontMaxTokens ? 4 : 6;
}

}  // extern "C"
