// Shared constants and sm_100a device primitives for the fused FP8 block-scale
// DeepSeek-V3 MoE layer (definition moe_fp8_block_scale_ds_routing_topk8_ng8_kg4
// _e32_h7168_i2048; shape constants as in the reference solution/python/kernel.h:10-25,
// except that the number of local experts is a runtime value here).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "../../include/moe_fp8_ds.h"

namespace moe {

constexpr int kHidden = 7168;            // H
constexpr int kInter = 2048;             // I
constexpr int kGemm1Out = 2 * kInter;    // 4096 rows of W13 per expert
constexpr int kBlock = 128;              // quantisation block (1x128 activations, 128x128 weights)
constexpr int kHiddenBlocks = kHidden / kBlock;   // 56
constexpr int kInterBlocks = kInter / kBlock;     // 16
constexpr int kExpertsGlobal = 256;
constexpr int kTopK = 8;
constexpr int kGroups = 8;
constexpr int kTopKGroups = 4;
constexpr int kGroupSize = kExpertsGlobal / kGroups;   // 32
constexpr float kFp8Max = 448.0f;

// Permutation block: tokens per routing CTA (one warp per token); the
// per-block expert masks are 32-bit.
constexpr int kPermBlock = 32;
// Tokens routed per CTA (one warp each); four route CTAs make a permutation block.
constexpr int kRouteTokens = 8;
// Largest batch served by the single-launch front end (32 CTAs of 8 tokens).
constexpr int kFrontMaxTokens = 256;

// A bounded wait gives up after this many nanoseconds and raises the
// device error word; every kernel here finishes in well under a second.
constexpr unsigned long long kWaitLimitNs = 1000ull * 1000ull * 1000ull;

// Device error word codes (written with atomicCAS so the first error wins).
enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutProducer = 1,
  kDevTimeoutMma = 2,
  kDevTimeoutEpilogue = 3,
  kDevBadExpertId = 4,
  kDevCapacity = 5,
  kDevTimeoutBarrier = 6,
};

// --------------------------------------------------------------------------
// Small PTX helpers
// --------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void raise_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ---- programmatic dependent launch --------------------------------------
// Wait until the preceding kernel in the stream has completed and its writes
// are visible (no-op when launched without the PDL attribute).
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Allow the next kernel in the stream to begin launching its CTAs.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- cross-CTA flags -------------------------------------------------------
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Counter updates that publish (release) and read (acquire) the data a CTA
// wrote before them.  Used after a CTA-wide barrier by one thread: the barrier
// orders the other threads' stores before the release (cumulativity), so one
// signalling thread replaces a fence in every thread.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void red_add_release_gpu(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Order this thread's earlier (generic-proxy) observations before its later
// async-proxy (TMA) accesses.
// Work unit u of a grouped GEMM -> (token tile mt, weight tile nt), token-tile
// major: the CTAs running at the same time cover a few token tiles with all of
// their weight tiles, so the two or three token tiles of one expert read each
// weight tile from L2 rather than from HBM again, and each expert's tiles finish
// together (the early-start consumer waits per expert).
__host__ __device__ __forceinline__ int2 unit_tile(int u, int n_mt, int NT) {
  (void)n_mt;
  return make_int2(u / NT, u % NT);
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async;" ::: "memory");
}
// Spin (bounded) until *ctr >= target; false on timeout or when another role
// has aborted.
__device__ __forceinline__ bool wait_counter(const int* ctr, int target, volatile int* abort_flag) {
  if (ld_acquire_gpu(ctr) >= target) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (ld_acquire_gpu(ctr) < target) {
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) { *abort_flag = 1; return false; }
    __nanosleep(128);
  }
  return true;
}

// ---- mbarrier -------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the phase with the given parity has completed.  Gives up (and
// sets *abort) after kWaitLimitNs, or as soon as another role has aborted.
// The clock and the abort flag are checked once per 64 polls: reading
// %globaltimer between polls delayed the wake-up after a phase completed by
// up to a microsecond on B200.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int k = 0; k < 64; ++k)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      *abort_flag = 1;
      return false;
    }
  }
}

// Warp-uniform form of mbar_wait_bounded for code that follows with
// .sync.aligned instructions (tcgen05.ld): lane 0 waits, every lane gets its
// result, and the warp is converged on return.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait_bounded(bar, parity, abort_flag) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

// ---- TMA ------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 3D tiled load: x = byte inside a 128-byte K block, y = row, z = K block.
__device__ __forceinline__ void tma_load_3d(const CUtensorMap* map, uint64_t* bar, void* smem_dst,
                                            int32_t x, int32_t y, int32_t z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}

// Row gather (tile::gather4) of a 2D K-major e4m3 matrix whose tensor map
// box is 128 bytes x 1 row: rows r0..r3, bytes x..x+127 (x a multiple of
// 128), landing as four consecutive 128-byte-swizzled rows at smem_dst.
__device__ __forceinline__ void tma_gather4(const CUtensorMap* map, uint64_t* bar, void* smem_dst, int32_t x,
                                            int32_t r0, int32_t r1, int32_t r2, int32_t r3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4, %5, %6, %7}], [%2], %8;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(r0), "r"(r1), "r"(r2), "r"(r3),
      "l"(policy)
      : "memory");
}

// 2D tiled load: x = innermost element index (its byte offset must be a
// multiple of 16), y = row.
__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* smem_dst,
                                            int32_t x, int32_t y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// 4D tiled load (coordinates innermost first).
__device__ __forceinline__ void tma_load_4d(const CUtensorMap* map, uint64_t* bar, void* smem_dst,
                                            int32_t x, int32_t y, int32_t z, int32_t w, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- tcgen05 / TMEM -------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrive on an mbarrier once all tcgen05 operations issued so far by this thread completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, e4m3 x e4m3 -> f32, both operands K-major.
__device__ __forceinline__ void tc_mma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor for kind::f8f6f4: A=B=e4m3, D=f32, K-major A and B, M=128.
__host__ __device__ constexpr uint32_t make_idesc_f8(int m, int n) {
  return (1u << 4)                            // D format f32
         | (0u << 7) | (0u << 10)             // A, B format e4m3
         | (0u << 15) | (0u << 16)            // A, B K-major
         | ((uint32_t)(n >> 3) << 17)         // N / 8
         | ((uint32_t)(m >> 4) << 24);        // M / 16
}

// Shared-memory matrix descriptor for a K-major tile written by TMA with
// 128-byte swizzling: rows of 128 bytes, 8-row core groups 1024 bytes apart.
__device__ __forceinline__ uint64_t make_sdesc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFF) >> 4);     // start address
  d |= (uint64_t)1 << 16;                          // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024 >> 4) << 32;                // stride byte offset: 8 rows * 128 B
  d |= (uint64_t)1 << 46;                          // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                          // layout: 128-byte swizzle
  return d;
}

// 32 lanes x 32 bits, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 bits, 32 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Load `cols` (16 or 32) consecutive TMEM columns.
template <int COLS>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float* v) {
  if constexpr (COLS == 32) tmem_ld32(taddr, v); else tmem_ld16(taddr, v);
}

// Barrier over `nthreads` threads that also ORs a per-thread flag; every
// thread gets the same result (used to take abort decisions uniformly).
__device__ __forceinline__ bool named_bar_or(int id, int nthreads, bool flag) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %2, 0;\n\t"
      "bar.red.or.pred q, %1, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out) : "r"(id), "r"((uint32_t)flag), "r"(nthreads) : "memory");
  return out != 0;
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Named barrier over a subset of warps (id 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ uint32_t elect_one_lane() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred;
}

// fp32 -> e4m3 with round-to-nearest-even and saturation to +-448.
__device__ __forceinline__ uint8_t f32_to_e4m3(float x) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}
__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
  __half_raw hr = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3);
  return __half2float(__half(hr));
}

// Launch with the programmatic-stream-serialization attribute (PDL).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
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
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace moe
