// Expert-parallel plumbing: dispatch planning, row packing/unpacking and the
// fixed-order combine, as device kernels behind the C ABI.
//
// The reference has no multi-GPU path; its only hook is local_expert_offset
// (solution/python/kernel.py:104).  Here rank r of `world` owns global experts
// [r*E_r, (r+1)*E_r).  A token's row goes once to every rank owning at least
// one of its 8 experts.  Send rows are ordered by (destination rank, token),
// and a row is
//   hidden e4m3 [7168] | scales fp32 [56] | expert ids int32 [8] | weights fp32 [8]
// (7456 bytes, every field 16-byte aligned).  The combine adds the partial
// rows that come back in ascending rank order in fp32 and rounds to bf16 once,
// so the result does not depend on message timing.
#include "kernels.cuh"

namespace moe {

constexpr int kRowBytes = kHidden + kHiddenBlocks * 4 + kTopK * 4 + kTopK * 4;   // 7456
constexpr int kOffScale = kHidden;
constexpr int kOffIds = kOffScale + kHiddenBlocks * 4;
constexpr int kOffW = kOffIds + kTopK * 4;
static_assert(kRowBytes == 7456 && kOffIds % 16 == 0 && kOffW % 16 == 0, "row layout");
constexpr int kMaxWorld = 8;

// One CTA.  Pass 1 counts the rows each rank receives; pass 2 gives every
// (token, rank) pair its send row: rank base + rank of the token among that
// rank's tokens.  Compact layout (cap = 0): rank bases are the prefix sums of
// the counts.  Fixed-capacity layout (cap >= T): rank r's rows start at
// r * cap and the unused rows of its block are padding (src_token = -1), so
// every all-to-all moves cap rows per peer and no count leaves the device.
__global__ void __launch_bounds__(1024) ep_plan_kernel(const int32_t* __restrict__ ids, int T, int world,
                                                        int experts_per_rank, int cap, int64_t* __restrict__ counts,
                                                        int32_t* __restrict__ slot, int32_t* __restrict__ src_token) {
  __shared__ int s_warp[32][kMaxWorld];
  __shared__ int s_run[kMaxWorld];
  __shared__ int s_base[kMaxWorld];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  auto dest_mask = [&](int t) -> uint32_t {
    uint32_t m = 0;
    if (t < T) {
#pragma unroll
      for (int k = 0; k < kTopK; ++k) {
        const int e = __ldg(ids + (size_t)t * kTopK + k);
        if (e >= 0 && e < experts_per_rank * world) m |= 1u << (e / experts_per_rank);
      }
    }
    return m;
  };
  if (tid < kMaxWorld) s_run[tid] = 0;
  __syncthreads();
  // pass 1: per-rank totals
  for (int c0 = 0; c0 < T; c0 += blockDim.x) {
    const uint32_t m = dest_mask(c0 + tid);
    for (int r = 0; r < world; ++r) {
      const uint32_t b = __ballot_sync(0xffffffffu, (m >> r) & 1u);
      if (lane == 0) atomicAdd(&s_run[r], __popc(b));
    }
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int r = 0; r < world; ++r) {
      s_base[r] = cap > 0 ? r * cap : acc;
      counts[r] = s_run[r];
      acc += s_run[r];
    }
  }
  __syncthreads();
  if (cap > 0)   // padding rows of every rank's block
    for (int r = 0; r < world; ++r)
      for (int j = s_run[r] + tid; j < cap; j += blockDim.x) src_token[r * cap + j] = -1;
  if (tid < kMaxWorld) s_run[tid] = 0;
  __syncthreads();
  // pass 2: slots, in token order inside each rank
  for (int c0 = 0; c0 < T; c0 += blockDim.x) {
    const int t = c0 + tid;
    const uint32_t m = dest_mask(t);
    uint32_t below[kMaxWorld];
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r) {
      if (r >= world) break;
      const uint32_t b = __ballot_sync(0xffffffffu, (m >> r) & 1u);
      below[r] = __popc(b & ((1u << lane) - 1u));
      if (lane == 0) s_warp[warp][r] = __popc(b);
    }
    __syncthreads();
    if (tid < world) {   // exclusive scan over warps, per rank
      int run = s_run[tid];
      for (int w = 0; w < 32; ++w) {
        const int v = s_warp[w][tid];
        s_warp[w][tid] = run;
        run += v;
      }
      s_run[tid] = run;
    }
    __syncthreads();
    if (t < T) {
#pragma unroll
      for (int r = 0; r < kMaxWorld; ++r) {
        if (r >= world) break;
        int32_t row = -1;
        if ((m >> r) & 1u) {
          row = s_base[r] + s_warp[warp][r] + (int)below[r];
          src_token[row] = t;
        }
        slot[(size_t)t * world + r] = row;
      }
    }
    __syncthreads();
  }
}

// A padding row (src_token < 0, fixed-capacity layout) is zero, with all 8
// expert ids set to the first expert of the next rank: a valid id that the
// receiving rank (row / cap) does not own, so its layer gives the row no work
// and a zero partial.
__global__ void __launch_bounds__(256) ep_pack_kernel(const int32_t* __restrict__ ids, const float* __restrict__ w,
                                                       const uint8_t* __restrict__ hidden,
                                                       const float* __restrict__ hidden_scale, int T,
                                                       const int32_t* __restrict__ src_token, int cap, int world,
                                                       int experts_per_rank, uint8_t* __restrict__ send) {
  const int row = blockIdx.x;
  const int t = __ldg(src_token + row);
  uint8_t* dst = send + (size_t)row * kRowBytes;
  if (t < 0) {
    const int foreign = ((row / cap + 1) % world) * experts_per_rank;
    for (int j = threadIdx.x; j < kOffIds / 16; j += blockDim.x)
      reinterpret_cast<uint4*>(dst)[j] = make_uint4(0u, 0u, 0u, 0u);
    const int j = threadIdx.x;
    if (j < kTopK) reinterpret_cast<int32_t*>(dst + kOffIds)[j] = foreign;
    else if (j < 2 * kTopK) reinterpret_cast<float*>(dst + kOffW)[j - kTopK] = 0.f;
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(hidden + (size_t)t * kHidden);
  for (int j = threadIdx.x; j < kHidden / 16; j += blockDim.x)
    reinterpret_cast<uint4*>(dst)[j] = __ldg(src + j);
  const int j = threadIdx.x;
  if (j < kHiddenBlocks)
    reinterpret_cast<float*>(dst + kOffScale)[j] = __ldg(hidden_scale + (size_t)j * T + t);
  else if (j >= 64 && j < 64 + kTopK)
    reinterpret_cast<int32_t*>(dst + kOffIds)[j - 64] = __ldg(ids + (size_t)t * kTopK + (j - 64));
  else if (j >= 96 && j < 96 + kTopK)
    reinterpret_cast<float*>(dst + kOffW)[j - 96] = __ldg(w + (size_t)t * kTopK + (j - 96));
}

__global__ void __launch_bounds__(256) ep_unpack_kernel(const uint8_t* __restrict__ recv, int R,
                                                         uint8_t* __restrict__ hidden, float* __restrict__ hidden_scale,
                                                         int32_t* __restrict__ ids, float* __restrict__ w) {
  const int row = blockIdx.x;
  const uint8_t* src = recv + (size_t)row * kRowBytes;
  uint4* dst = reinterpret_cast<uint4*>(hidden + (size_t)row * kHidden);
  for (int j = threadIdx.x; j < kHidden / 16; j += blockDim.x)
    dst[j] = reinterpret_cast<const uint4*>(src)[j];
  const int j = threadIdx.x;
  if (j < kHiddenBlocks)
    hidden_scale[(size_t)j * R + row] = reinterpret_cast<const float*>(src + kOffScale)[j];
  else if (j >= 64 && j < 64 + kTopK)
    ids[(size_t)row * kTopK + (j - 64)] = reinterpret_cast<const int32_t*>(src + kOffIds)[j - 64];
  else if (j >= 96 && j < 96 + kTopK)
    w[(size_t)row * kTopK + (j - 96)] = reinterpret_cast<const float*>(src + kOffW)[j - 96];
}

// out[t] = bf16( sum over r ascending, slot[t][r] >= 0, of float(part[slot[t][r]]) ),
// the sum starting from +0.  Grid (T, 7); 128 threads x 8 columns.
// Partials arrive in fp32 (each rank's sum over its own picks, not rounded),
// so the only rounding to bf16 is the final one, as on one GPU.
__global__ void __launch_bounds__(128) ep_combine_kernel(const float* __restrict__ part,
                                                          const int32_t* __restrict__ slot, int world,
                                                          __nv_bfloat16* __restrict__ out) {
  const int t = blockIdx.x;
  const int col = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  float acc[8];
#pragma unroll
  for (int x = 0; x < 8; ++x) acc[x] = 0.f;
  for (int r = 0; r < world; ++r) {
    const int s = __ldg(slot + (size_t)t * world + r);
    if (s < 0) continue;
    const float4* src = reinterpret_cast<const float4*>(part + (size_t)s * kHidden + col);
    const float4 a = __ldg(src), b = __ldg(src + 1);
    acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
    acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
  }
  uint4 o;
  __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
  for (int x = 0; x < 4; ++x) oh[x] = __floats2bfloat162_rn(acc[2 * x], acc[2 * x + 1]);
  *reinterpret_cast<uint4*>(out + (size_t)t * kHidden + col) = o;
}

namespace {
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
int launch_status() { return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA; }
}  // namespace

}  // namespace moe

using namespace moe;

extern "C" {

MOE_API int moe_fp8_ds_ep_plan(const int32_t* topk_ids, int32_t num_tokens, int32_t world,
                               int32_t experts_per_rank, int64_t* counts, int32_t* slot,
                               int32_t* src_token, void* stream) {
  if (num_tokens < 0 || world < 1 || world > kMaxWorld || experts_per_rank < 1 ||
      experts_per_rank * world != kExpertsGlobal || !counts)
    return MOE_ERR_INVALID_ARGUMENT;
  if (num_tokens > 0 && (!topk_ids || !slot || !src_token)) return MOE_ERR_INVALID_ARGUMENT;
  ep_plan_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(topk_ids, num_tokens, world,
                                                                     experts_per_rank, 0, counts, slot, src_token);
  return launch_status();
}

MOE_API int moe_fp8_ds_ep_plan_capacity(const int32_t* topk_ids, int32_t num_tokens, int32_t world,
                                        int32_t experts_per_rank, int32_t capacity, int64_t* counts,
                                        int32_t* slot, int32_t* src_token, void* stream) {
  if (num_tokens < 0 || world < 2 || world > kMaxWorld || experts_per_rank < 1 ||
      experts_per_rank * world != kExpertsGlobal || !counts || capacity < num_tokens || capacity < 1)
    return MOE_ERR_INVALID_ARGUMENT;
  if (!src_token || (num_tokens > 0 && (!topk_ids || !slot))) return MOE_ERR_INVALID_ARGUMENT;
  ep_plan_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(topk_ids, num_tokens, world,
                                                                     experts_per_rank, capacity, counts, slot,
                                                                     src_token);
  return launch_status();
}

MOE_API int moe_fp8_ds_ep_pack(const int32_t* topk_ids, const float* topk_weights, const void* hidden_states,
                               const float* hidden_states_scale, int32_t num_tokens, const int32_t* src_token,
                               int32_t rows, void* send, void* stream) {
  if (num_tokens < 0 || rows < 0) return MOE_ERR_INVALID_ARGUMENT;
  if (rows == 0) return MOE_OK;
  if (!topk_ids || !topk_weights || !hidden_states || !hidden_states_scale || !src_token || !send)
    return MOE_ERR_INVALID_ARGUMENT;
  if (!aligned16(hidden_states) || !aligned16(send)) return MOE_ERR_MISALIGNED;
  ep_pack_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      topk_ids, topk_weights, static_cast<const uint8_t*>(hidden_states), hidden_states_scale, num_tokens,
      src_token, 1, 1, kExpertsGlobal, static_cast<uint8_t*>(send));
  return launch_status();
}

MOE_API int moe_fp8_ds_ep_pack_capacity(const int32_t* topk_ids, const float* topk_weights,
                                        const void* hidden_states, const float* hidden_states_scale,
                                        int32_t num_tokens, const int32_t* src_token, int32_t world,
                                        int32_t experts_per_rank, int32_t capacity, void* send, void* stream) {
  if (num_tokens < 0 || world < 2 || world > kMaxWorld || experts_per_rank * world != kExpertsGlobal ||
      capacity < num_tokens || capacity < 1)
    return MOE_ERR_INVALID_ARGUMENT;
  if (!src_token || !send || (num_tokens > 0 && (!topk_ids || !topk_weights || !hidden_states ||
                                                 !hidden_states_scale)))
    return MOE_ERR_INVALID_ARGUMENT;
  if ((hidden_states && !aligned16(hidden_states)) || !aligned16(send)) return MOE_ERR_MISALIGNED;
  ep_pack_kernel<<<world * capacity, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      topk_ids, topk_weights, static_cast<const uint8_t*>(hidden_states), hidden_states_scale, num_tokens,
      src_token, capacity, world, experts_per_rank, static_cast<uint8_t*>(send));
  return launch_status();
}

MOE_API int moe_fp8_ds_ep_unpack(const void* recv, int32_t rows, void* hidden_states, float* hidden_states_scale,
                                 int32_t* topk_ids, float* topk_weights, void* stream) {
  if (rows < 0) return MOE_ERR_INVALID_ARGUMENT;
  if (rows == 0) return MOE_OK;
  if (!recv || !hidden_states || !hidden_states_scale || !topk_ids || !topk_weights)
    return MOE_ERR_INVALID_ARGUMENT;
  if (!aligned16(recv) || !aligned16(hidden_states)) return MOE_ERR_MISALIGNED;
  ep_unpack_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(recv), rows, static_cast<uint8_t*>(hidden_states), hidden_states_scale,
      topk_ids, topk_weights);
  return launch_status();
}

MOE_API int moe_fp8_ds_ep_combine(const void* partials, const int32_t* slot, int32_t num_tokens, int32_t world,
                                  void* output, void* stream) {
  if (num_tokens < 0 || world < 1 || world > kMaxWorld) return MOE_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return MOE_OK;
  if (!slot || !output) return MOE_ERR_INVALID_ARGUMENT;
  if (!aligned16(output) || (partials && !aligned16(partials))) return MOE_ERR_MISALIGNED;
  ep_combine_kernel<<<dim3(num_tokens, kHidden / (128 * 8)), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const float*>(partials), slot, world, static_cast<__nv_bfloat16*>(output));
  return launch_status();
}

}  // extern "C"
