// Routing, token->expert permutation and weighted combine for the fused FP8
// DeepSeek-V3 MoE layer.  All kernels here are SIMT and HBM/latency bound;
// the GEMMs live in gemm_fp8.cu.
//
// Reference behaviour followed:
//   routing   solution/python/kernel.cu:56-200 (CUDA), solution/cuda/moe.cu:178-206
//             (ATen) and flashinfer trace/templates/moe.py:140-170 (contest definition)
//   permute   solution/python/kernel.cu:321-351, 503-537, 676-741, 1344-1368, 204-218
//   combine   solution/python/kernel.cu:809-839 (deterministic finalize)
#include "kernels.cuh"

namespace moe {

// --------------------------------------------------------------------------
// Routing + per-block token masks of local experts.
//
// One warp per token, 32 tokens per CTA ("permutation block"); lane l owns
// experts 8l..8l+7, so routing group g is lanes 4g..4g+3.  Arithmetic mirrors
// the reference definition:
//   s  = 1 / (1 + exp(-x))        exp correctly rounded (evaluated in fp64)
//   sb = s + bias
//   group score = sum of the two largest sb in the group; keep the best 4
//   top-8 of sb inside kept groups
//   w_k = (s_k / (sum_s + 1e-20)) * routed_scaling_factor
// The normaliser sum_s adds the selected s values in the order torch's CPU
// row reduction uses for a [T,256] fp32 tensor (8 lanes of 4 interleaved
// accumulators, lanes summed last), so weights match the reference's own
// fp32 arithmetic.  Ties in any top-k go to the lower index.
//
// One CTA routes kRouteTokens tokens and writes the byte masks8[e][g], bit
// w set when token 8g+w picked local expert e (rows of NB8p = 4*ceil(T/32)
// bytes, zero-padded).  Four consecutive bytes form the 32-token
// permutation-block mask that the scan turns into row offsets and the scatter
// into each token's rank inside its expert (ascending tokens).
// --------------------------------------------------------------------------
// Routes token t with one warp; returns the token's k-th expert id (ascending)
// in lane k < 8 and -1 elsewhere, and writes ids/weights unless kFromIds.
template <bool kFromIds>
__device__ __forceinline__ int route_token(int t, int lane, const float* __restrict__ logits,
                                           const __nv_bfloat16* __restrict__ bias, float scaling,
                                           int32_t* __restrict__ topk_ids, float* __restrict__ topk_w,
                                           int* __restrict__ err) {
  int my_id = -1;  // lane k < 8 ends up holding the k-th id (ascending)
  if constexpr (!kFromIds) {
    const float4* lp = reinterpret_cast<const float4*>(logits + (size_t)t * kExpertsGlobal) + lane * 2;
    float4 l0 = lp[0], l1 = lp[1];
    float x[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
    uint4 braw = reinterpret_cast<const uint4*>(bias)[lane];
    const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(&braw);
    float s[8], sb[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float e = (float)exp(-(double)x[j]);
      s[j] = __frcp_rn(__fadd_rn(1.0f, e));
      sb[j] = __fadd_rn(s[j], __bfloat162float(bb[j]));
    }
    // ---- group score: sum of the top-2 sb of each 32-expert group
    float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float v = sb[j];
      if (v > m1) { m2 = m1; m1 = v; } else if (v > m2) { m2 = v; }
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      float o1 = __shfl_xor_sync(0xffffffffu, m1, off);
      float o2 = __shfl_xor_sync(0xffffffffu, m2, off);
      float n1, n2;
      if (m1 >= o1) { n1 = m1; n2 = fmaxf(m2, o1); } else { n1 = o1; n2 = fmaxf(m1, o2); }
      m1 = n1; m2 = n2;
    }
    const float gscore = __fadd_rn(m1, m2);
    // ---- keep the best 4 groups (ties: lower group)
    float gs[kGroups];
#pragma unroll
    for (int g = 0; g < kGroups; ++g) gs[g] = __shfl_sync(0xffffffffu, gscore, 4 * g);
    unsigned keep = 0;
#pragma unroll
    for (int r = 0; r < kTopKGroups; ++r) {
      int best = -1; float bv = -INFINITY;
#pragma unroll
      for (int g = 0; g < kGroups; ++g)
        if (!((keep >> g) & 1u) && (best < 0 || gs[g] > bv)) { best = g; bv = gs[g]; }
      keep |= 1u << best;
    }
    const bool my_group_kept = (keep >> (lane >> 2)) & 1u;
    // ---- top-8 experts of sb inside kept groups.  Each lane keeps the index
    // of its best untaken candidate (lowest j on ties); a round takes the
    // warp-wide maximum with one redux on an order-preserving integer key,
    // and the lowest lane holding it (= lowest expert id on ties) gives it up.
    auto key_of = [](float v) -> uint32_t {   // monotone float -> u32
      const uint32_t b = __float_as_uint(v);
      return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    };
    float cand[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) cand[j] = my_group_kept ? sb[j] : -INFINITY;
    unsigned taken = 0;
    auto local_best = [&]() -> int {
      int bj = -1; float bv = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (!((taken >> j) & 1u) && (bj < 0 || cand[j] > bv)) { bj = j; bv = cand[j]; }
      return bj;
    };
    int bj = local_best();
    int sel_e[kTopK];
    float sel_s[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      float bv = -INFINITY, bs = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) if (j == bj) { bv = cand[j]; bs = s[j]; }
      const uint32_t key = bj < 0 ? 0u : key_of(bv);
      const uint32_t top = __reduce_max_sync(0xffffffffu, key);
      const uint32_t holders = __ballot_sync(0xffffffffu, key == top);
      const int wl = __ffs(holders) - 1;
      const int wj = __shfl_sync(0xffffffffu, bj, wl);
      sel_e[k] = wl * 8 + wj;
      sel_s[k] = __shfl_sync(0xffffffffu, bs, wl);
      if (lane == wl) {
        taken |= 1u << wj;
        bj = local_best();
      }
    }
    // ---- sort the 8 picks ascending (all lanes hold the same arrays)
#pragma unroll
    for (int a = 1; a < kTopK; ++a)
#pragma unroll
      for (int b = a; b > 0; --b)
        if (sel_e[b] < sel_e[b - 1]) {
          int te = sel_e[b]; sel_e[b] = sel_e[b - 1]; sel_e[b - 1] = te;
          float ts = sel_s[b]; sel_s[b] = sel_s[b - 1]; sel_s[b - 1] = ts;
        }
    // ---- normaliser in torch's CPU reduction order: lane l (< 8) forms the
    // vector-lane partial P_l = ((A0+A1)+A2)+A3 with A_q = sum (ascending
    // expert id) of picks e with e%8 == l and (e/8)%4 == q.
    float P = 0.f;
    if (lane < 8) {
      float A[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k < kTopK; ++k)
        if ((sel_e[k] & 7) == lane) {
          int q = (sel_e[k] >> 3) & 3;
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) if (qq == q) A[qq] = __fadd_rn(A[qq], sel_s[k]);
        }
      P = __fadd_rn(__fadd_rn(__fadd_rn(A[0], A[1]), A[2]), A[3]);
    }
    float total = 0.f;
#pragma unroll
    for (int l = 0; l < 8; ++l) total = __fadd_rn(total, __shfl_sync(0xffffffffu, P, l));
    const float denom = __fadd_rn(total, 1e-20f);
    if (lane < kTopK) {
      float my_w = 0.f; int my_e = 0;
#pragma unroll
      for (int k = 0; k < kTopK; ++k) if (k == lane) { my_e = sel_e[k]; my_w = sel_s[k]; }
      my_w = __fmul_rn(__fdiv_rn(my_w, denom), scaling);
      topk_ids[(size_t)t * kTopK + lane] = my_e;
      topk_w[(size_t)t * kTopK + lane] = my_w;
      my_id = my_e;
    }
  } else {
    if (lane < kTopK) {
      my_id = topk_ids[(size_t)t * kTopK + lane];
      if (my_id < 0 || my_id >= kExpertsGlobal) { raise_error(err, kDevBadExpertId); my_id = -1; }
    }
  }
  return my_id;
}

// CTA g stores its byte of every expert row; the last CTA zeroes the padding.
__device__ __forceinline__ void store_masks(uint8_t* __restrict__ masks8, int NB8p, int E_l,
                                            const uint32_t* s_mask) {
  for (int e = threadIdx.x; e < E_l; e += blockDim.x) {
    uint8_t* row = masks8 + (size_t)e * NB8p;
    row[blockIdx.x] = static_cast<uint8_t>(s_mask[e]);
    if (blockIdx.x == gridDim.x - 1)
      for (int g = gridDim.x; g < NB8p; ++g) row[g] = 0;
  }
}

template <bool kFromIds>
__global__ void __launch_bounds__(kRouteTokens * 32)
route_kernel(const float* __restrict__ logits, const __nv_bfloat16* __restrict__ bias,
             int T, float scaling, int local_offset, int E_l,
             int32_t* __restrict__ topk_ids, float* __restrict__ topk_w,
             uint8_t* __restrict__ masks8, int NB8p, int* __restrict__ err) {
  __shared__ uint32_t s_mask[kExpertsGlobal];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  griddep_wait();
  griddep_launch_dependents();
  for (int e = threadIdx.x; e < E_l; e += blockDim.x) s_mask[e] = 0;
  __syncthreads();

  const int t = blockIdx.x * kRouteTokens + warp;
  if (t < T) {
    const int my_id = route_token<kFromIds>(t, lane, logits, bias, scaling, topk_ids, topk_w, err);
    if (lane < kTopK && my_id >= 0) {
      int le = my_id - local_offset;
      if (le >= 0 && le < E_l) atomicOr(&s_mask[le], 1u << warp);
    }
  }
  __syncthreads();
  if (masks8) store_masks(masks8, NB8p, E_l, s_mask);
}

// 32-token block mask of block b for expert e from the four byte masks.
__device__ __forceinline__ uint32_t block_mask(const uint8_t* __restrict__ masks8, int NB8p, int E_l,
                                               int b, int e) {
  (void)E_l;
  return __ldcg(reinterpret_cast<const unsigned int*>(masks8 + (size_t)e * NB8p) + b);
}

// --------------------------------------------------------------------------
// Scan: per-expert row segments, per-(CTA, expert) row bases, GEMM tile
// lists, and zeroed stream-K counters.  One CTA of 1024 threads.
// --------------------------------------------------------------------------
// Token tile m of the n = ceil(cnt / bn) tiles of one expert's cnt rows.  The
// rows are split evenly (tile sizes differ by at most one) rather than as
// full tiles plus a remainder, so no tile is nearly empty: the GEMMs size the
// MMA's N to the tile, and an even split keeps that N small.
__device__ __forceinline__ int4 balanced_tile(int e, int r0, int cnt, int n, int m) {
  const int a = m * cnt / n, b = (m + 1) * cnt / n;
  return make_int4(e, r0 + a, b - a, 0);
}

__device__ __forceinline__ int warp_exclusive_scan(int v, int lane, int* total) {
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    int o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  if (total) *total = __shfl_sync(0xffffffffu, incl, 31);
  return incl - v;
}

// Exclusive scan of n <= 256 values in smem by warp 0 (8 per lane), result in place.
__device__ void warp0_scan_inplace(int* v, int n, int* total_out) {
  const int lane = threadIdx.x & 31;
  int loc[8];
  int sum = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int idx = lane * 8 + i;
    loc[i] = idx < n ? v[idx] : 0;
    sum += loc[i];
  }
  int total;
  int base = warp_exclusive_scan(sum, lane, &total);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int idx = lane * 8 + i;
    if (idx < n) v[idx] = base;
    base += loc[i];
  }
  if (lane == 0 && total_out) *total_out = total;
}

__global__ void __launch_bounds__(1024)
scan_kernel(const uint8_t* __restrict__ masks8, int NB8p, int32_t* __restrict__ bases, int NB, int E_l,
            int32_t* __restrict__ seg_out,
            int bn1, int bn2, int4* __restrict__ tiles1, int4* __restrict__ tiles2,
            int32_t* __restrict__ sched, int32_t* __restrict__ counters1, int nt1,
            int32_t* __restrict__ counters2, int nt2, int* __restrict__ ready) {
  __shared__ int s_cnt[kExpertsGlobal];
  __shared__ int s_seg[kExpertsGlobal + 1];
  __shared__ int s_t1[kExpertsGlobal];
  __shared__ int s_t2[kExpertsGlobal];
  __shared__ int s_tot[3];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;

  griddep_wait();
  griddep_launch_dependents();
  // 1. per-expert totals and per-(block, expert) exclusive bases
  for (int e = warp; e < E_l; e += nwarps) {
    int run = 0;
    for (int b0 = 0; b0 < NB; b0 += 32) {
      int b = b0 + lane;
      int v = b < NB ? __popc(block_mask(masks8, NB8p, E_l, b, e)) : 0;
      int tot;
      int ex = warp_exclusive_scan(v, lane, &tot);
      if (b < NB) bases[(size_t)b * E_l + e] = run + ex;   // relative to segment start
      run += tot;
    }
    if (lane == 0) s_cnt[e] = run;
  }
  __syncthreads();
  if (warp == 0) {
    for (int e = lane; e < E_l; e += 32) { s_seg[e] = s_cnt[e]; }
    __syncwarp();
    int tot;
    warp0_scan_inplace(s_seg, E_l, &tot);
    if (lane == 0) { s_seg[E_l] = tot; s_tot[0] = tot; }
  } else if (warp == 1) {
    for (int e = lane; e < E_l; e += 32) s_t1[e] = (s_cnt[e] + bn1 - 1) / bn1;
    __syncwarp();
    int tot;
    warp0_scan_inplace(s_t1, E_l, &tot);
    if (lane == 0) s_tot[1] = tot;
  } else if (warp == 2) {
    for (int e = lane; e < E_l; e += 32) s_t2[e] = (s_cnt[e] + bn2 - 1) / bn2;
    __syncwarp();
    int tot;
    warp0_scan_inplace(s_t2, E_l, &tot);
    if (lane == 0) s_tot[2] = tot;
  }
  __syncthreads();
  // 2. absolute bases, segment offsets, tile lists
  for (int i = threadIdx.x; i < NB * E_l; i += blockDim.x) bases[i] += s_seg[i % E_l];
  for (int e = threadIdx.x; e <= E_l; e += blockDim.x) seg_out[e] = s_seg[e];
  for (int e = warp; e < E_l; e += nwarps) {
    const int cnt = s_cnt[e], r0 = s_seg[e];
    const int n1 = (cnt + bn1 - 1) / bn1, n2 = (cnt + bn2 - 1) / bn2;
    for (int m = lane; m < n1; m += 32)
      tiles1[s_t1[e] + m] = balanced_tile(e, r0, cnt, n1, m);
    for (int m = lane; m < n2; m += 32)
      tiles2[s_t2[e] + m] = balanced_tile(e, r0, cnt, n2, m);
  }
  const int units1 = s_tot[1] * nt1, units2 = s_tot[2] * nt2;
  for (int i = threadIdx.x; i < units1; i += blockDim.x) counters1[i] = 0;
  for (int i = threadIdx.x; i < units2; i += blockDim.x) counters2[i] = 0;
  for (int e = threadIdx.x; e < E_l; e += blockDim.x) ready[e] = 0;
  if (threadIdx.x == 0) {
    sched[0] = s_tot[1];
    sched[1] = s_tot[2];
    sched[2] = s_tot[0];
  }
}

// --------------------------------------------------------------------------
// Scatter + gather: rows of local expert e are its tokens in ascending order;
// the rank of token 32b+w inside expert e is popc(masks[b][e] & ((1<<w)-1)).
// CTA (b, c) handles the 32 tokens of block b and copies the 256-byte column
// chunk c (two 128-wide K blocks) of each of their local rows into the
// permuted activation act[R_cap, 7168], with the two matching scales; chunk
// 0 also writes inv_row[t,k] (row or -1) and row_token[row].
// --------------------------------------------------------------------------
constexpr int kGatherChunk = 256;                          // bytes per CTA column chunk
constexpr int kGatherChunks = kHidden / kGatherChunk;      // 28

__global__ void __launch_bounds__(kPermBlock * kTopK)
scatter_kernel(const int32_t* __restrict__ topk_ids, const uint8_t* __restrict__ masks8, int NB8p,
               const int32_t* __restrict__ bases, int T, int E_l, int local_offset, int R_cap,
               const uint8_t* __restrict__ hidden, const float* __restrict__ hs_scale,
               int32_t* __restrict__ inv_row, int32_t* __restrict__ row_token,
               uint8_t* __restrict__ act, float* __restrict__ act_scale) {
  __shared__ int s_row[kPermBlock * kTopK];
  griddep_wait();
  griddep_launch_dependents();
  const int i = blockIdx.x * kPermBlock * kTopK + threadIdx.x;   // (t, k) pair
  const int t = i / kTopK;
  int row = -1;
  if (t < T) {
    const int le = topk_ids[i] - local_offset;
    if (le >= 0 && le < E_l) {
      const int w = t - blockIdx.x * kPermBlock;
      const size_t be = (size_t)blockIdx.x * E_l + le;
      row = bases[be] + __popc(block_mask(masks8, NB8p, E_l, blockIdx.x, le) & ((1u << w) - 1u));
    }
    if (blockIdx.y == 0) {
      inv_row[i] = row;
      if (row >= 0) row_token[row] = t;
    }
  }
  s_row[threadIdx.x] = row;
  // local (row, token) pairs, compacted (their order does not matter)
  __shared__ int2 s_list[kPermBlock * kTopK];
  __shared__ int s_n;
  if (threadIdx.x == 0) s_n = 0;
  __syncthreads();
  {
    const uint32_t m = __ballot_sync(0xffffffffu, row >= 0);
    int base = 0;
    if ((threadIdx.x & 31) == 0 && m) base = atomicAdd(&s_n, __popc(m));
    base = __shfl_sync(0xffffffffu, base, 0);
    if (row >= 0) s_list[base + __popc(m & ((1u << (threadIdx.x & 31)) - 1u))] = make_int2(row, t);
  }
  __syncthreads();
  // copy: 16-byte vectors of the compacted pairs, kBatch loads in flight per
  // thread before the stores
  constexpr int kVec = kGatherChunk / 16;
  constexpr int kBatch = 4;
  const size_t col = (size_t)blockIdx.y * kGatherChunk;
  const int nvec = s_n * kVec;
  for (int v0 = threadIdx.x; v0 < nvec; v0 += kBatch * blockDim.x) {
    uint4 val[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int v = v0 + u * blockDim.x;
      if (v < nvec) {
        const int2 rt = s_list[v / kVec];
        val[u] = __ldg(reinterpret_cast<const uint4*>(hidden + (size_t)rt.y * kHidden + col + (v % kVec) * 16));
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int v = v0 + u * blockDim.x;
      if (v >= nvec) break;
      const int2 rt = s_list[v / kVec];
      *reinterpret_cast<uint4*>(act + (size_t)rt.x * kHidden + col + (v % kVec) * 16) = val[u];
    }
  }
  const int r = s_row[threadIdx.x];
  if (r >= 0) {
    const int kb0 = blockIdx.y * (kGatherChunk / kBlock);
#pragma unroll
    for (int q = 0; q < kGatherChunk / kBlock; ++q)
      act_scale[(size_t)(kb0 + q) * R_cap + r] = __ldg(hs_scale + (size_t)(kb0 + q) * T + t);
  }
}

// --------------------------------------------------------------------------
// Fused front end for small batches (T <= kFrontMaxTokens): routing, row
// assignment and the activation scales in ONE launch instead of three (the
// token rows are gathered by GEMM1 itself, tile::gather4 from hidden_states).
//
// CTA g routes tokens 8g..8g+7 (one warp each) and publishes its byte masks;
// after a grid-wide barrier every CTA recomputes the per-expert row offsets
// from all masks (at most 32 x E_l bytes, cheaper than another launch), then
// assigns rows to its own tokens (inverse map, row -> token map) and copies
// their 1x128 scales into the permuted scale array.  CTA 0 also writes the segment offsets, the GEMM
// tile lists and zeroes the stream-K counters.  All CTAs are resident (at
// most 32 small CTAs); the barrier wait is bounded and raises the device error
// word instead of hanging.
// --------------------------------------------------------------------------
__device__ bool grid_barrier(int* count, volatile int* gen, int* err) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    const int g = *gen;
    __threadfence();
    if (atomicAdd(count, 1) == (int)gridDim.x - 1) {
      atomicExch(count, 0);
      __threadfence();
      atomicAdd(const_cast<int*>(gen), 1);
    } else {
      const unsigned long long t0 = globaltimer_ns();
      while (*gen == g) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) { ok = 0; raise_error(err, kDevTimeoutBarrier); break; }
        // spin: the waiting is short and its latency is on the critical path
      }
    }
    __threadfence();
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

__global__ void __launch_bounds__(kRouteTokens * 32)
front_kernel(const float* __restrict__ logits, const __nv_bfloat16* __restrict__ bias, int T,
             float scaling, int local_offset, int E_l, int R_cap, int bn1, int bn2, int nt1, int nt2,
             const uint8_t* __restrict__ hidden, const float* __restrict__ hs_scale,
             int32_t* __restrict__ topk_ids, float* __restrict__ topk_w, uint8_t* __restrict__ masks8,
             int NB8p, int32_t* __restrict__ seg_out, int4* __restrict__ tiles1, int4* __restrict__ tiles2,
             int32_t* __restrict__ sched, int32_t* __restrict__ counters1,
             int32_t* __restrict__ counters2, int* __restrict__ ready, int32_t* __restrict__ inv_row,
             int32_t* __restrict__ row_token, uint8_t* __restrict__ act, float* __restrict__ act_scale,
             int* __restrict__ err, int* __restrict__ front_sync) {
  __shared__ uint32_t s_mask[kExpertsGlobal];
  __shared__ int s_seg[kExpertsGlobal + 1];
  __shared__ int s_base[kExpertsGlobal];
  __shared__ int s_t1[kExpertsGlobal], s_t2[kExpertsGlobal];
  __shared__ int2 s_list[kRouteTokens * kTopK];
  __shared__ int s_tot[3];
  __shared__ int s_n;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  griddep_wait();
  // GEMM1 is released only after the barrier below, so it cannot see the
  // previous call's flags: they are cleared (and fenced) before CTA 0 reaches
  // it, by a warp of CTA 0 that routes no token when there is one (the fence
  // then stays off the routing path), else by warp 0 after its token.
  const bool single = gridDim.x == 1;
  const int reset_warp = T < kRouteTokens ? kRouteTokens - 1 : 0;
  const bool resetter = blockIdx.x == 0 && threadIdx.x == reset_warp * 32;
  auto reset_flags = [&]() {
    front_sync[0] = 0;
    front_sync[1] = 0;
    __threadfence();
  };
  if (resetter && T < kRouteTokens) reset_flags();
  for (int e = threadIdx.x; e < E_l; e += blockDim.x) s_mask[e] = 0;
  if (threadIdx.x == 0) s_n = 0;
  __syncthreads();
  // ---- phase 1: route own tokens, publish masks
  const int t = blockIdx.x * kRouteTokens + warp;
  int my_id = -1;
  if (t < T) {
    my_id = route_token<false>(t, lane, logits, bias, scaling, topk_ids, topk_w, err);
    if (lane < kTopK && my_id >= 0) {
      const int le = my_id - local_offset;
      if (le >= 0 && le < E_l) atomicOr(&s_mask[le], 1u << warp);
    }
  }
  if (resetter && T >= kRouteTokens) reset_flags();
  __syncthreads();
  if (!single) store_masks(masks8, NB8p, E_l, s_mask);
  // Up to eight CTAs run as one thread-block cluster (launch attribute) and
  // meet at the hardware cluster barrier, which also orders their global
  // writes (release/acquire at cluster scope); larger grids use the bounded
  // software grid barrier.
  uint32_t nctas_in_cluster;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(nctas_in_cluster));
  if (single) {
    // one CTA: the masks stay in shared memory, no barrier beyond the block's
  } else if (nctas_in_cluster == gridDim.x) {
    __syncthreads();
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  } else if (!grid_barrier(err + 1, err + 2, err)) {
    return;
  }
  griddep_launch_dependents();
  // ---- phase 2: per-expert counts and this CTA's first row per expert
  for (int e = threadIdx.x; e < E_l; e += blockDim.x) {
    const unsigned int* row = reinterpret_cast<const unsigned int*>(masks8 + (size_t)e * NB8p);
    const int g0 = blockIdx.x;
    int before = 0, total = single ? __popc(s_mask[e]) : 0;
#pragma unroll
    for (int q = 0; q < kFrontMaxTokens / kPermBlock; ++q) {
      if (single || q * 4 >= NB8p) break;
      const uint32_t m = __ldcg(row + q);
      total += __popc(m);
      if (4 * q + 4 <= g0) before += __popc(m);
      else if (4 * q < g0) before += __popc(m & ((1u << (8 * (g0 - 4 * q))) - 1u));
    }
    s_seg[e] = total;
    s_base[e] = before;
    s_t1[e] = (total + bn1 - 1) / bn1;
    s_t2[e] = (total + bn2 - 1) / bn2;
  }
  __syncthreads();
  if (warp == 0) {
    int tot;
    warp0_scan_inplace(s_seg, E_l, &tot);
    if (lane == 0) { s_seg[E_l] = tot; s_tot[0] = tot; }
  } else if (warp == 1 && blockIdx.x == 0) {
    int tot;
    warp0_scan_inplace(s_t1, E_l, &tot);
    if (lane == 0) s_tot[1] = tot;
  } else if (warp == 2 && blockIdx.x == 0) {
    int tot;
    warp0_scan_inplace(s_t2, E_l, &tot);
    if (lane == 0) s_tot[2] = tot;
  }
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int e = threadIdx.x; e <= E_l; e += blockDim.x) seg_out[e] = s_seg[e];
    for (int e = warp; e < E_l; e += blockDim.x / 32) {
      const int cnt = s_seg[e + 1] - s_seg[e], r0 = s_seg[e];
      const int n1 = (cnt + bn1 - 1) / bn1, n2 = (cnt + bn2 - 1) / bn2;
      for (int m = lane; m < n1; m += 32)
        tiles1[s_t1[e] + m] = balanced_tile(e, r0, cnt, n1, m);
      for (int m = lane; m < n2; m += 32)
        tiles2[s_t2[e] + m] = balanced_tile(e, r0, cnt, n2, m);
    }
    const int units1 = s_tot[1] * nt1, units2 = s_tot[2] * nt2;
    for (int i = threadIdx.x; i < units1; i += blockDim.x) counters1[i] = 0;
    for (int i = threadIdx.x; i < units2; i += blockDim.x) counters2[i] = 0;
    for (int e = threadIdx.x; e < E_l; e += blockDim.x) ready[e] = 0;
    if (threadIdx.x == 0) { sched[0] = s_tot[1]; sched[1] = s_tot[2]; sched[2] = s_tot[0]; }
    __syncthreads();
    if (threadIdx.x == 0) {   // tile lists, schedule, counters published
      __threadfence();
      atomicExch(front_sync, 1);
    }
  }
  // ---- phase 3: rows of own tokens, inverse map, row -> token map, scales
  if (threadIdx.x < kRouteTokens * kTopK) {
    const int w8 = threadIdx.x / kTopK, k = threadIdx.x % kTopK;
    const int tt = blockIdx.x * kRouteTokens + w8;
    if (tt < T) {
      int row = -1;
      const int le = topk_ids[(size_t)tt * kTopK + k] - local_offset;
      if (le >= 0 && le < E_l) {
        row = s_seg[le] + s_base[le] + __popc(s_mask[le] & ((1u << w8) - 1u));
        row_token[row] = tt;
        s_list[atomicAdd(&s_n, 1)] = make_int2(row, tt);
      }
      inv_row[(size_t)tt * kTopK + k] = row;
    }
  }
  __syncthreads();
  // The token rows themselves are not copied: GEMM1 gathers them from
  // hidden_states by row_token (tile::gather4).  Their 1x128 scales are.
  for (int v = threadIdx.x; v < s_n * kHiddenBlocks; v += blockDim.x) {
    const int2 rt = s_list[v / kHiddenBlocks];
    const int kb = v % kHiddenBlocks;
    act_scale[(size_t)kb * R_cap + rt.x] = __ldg(hs_scale + (size_t)kb * T + rt.y);
  }
  __syncthreads();
  if (threadIdx.x == 0) {     // this CTA's rows of row_token / act_scale are written
    __threadfence();
    atomicAdd(front_sync + 1, 1);
  }
}

// --------------------------------------------------------------------------
// Combine: out[t] = sum_k w[t,k] * down[inv[t,k]] over local picks, in
// ascending expert order, fp32 multiply-then-add (as index_add_ does), then bf16.
// --------------------------------------------------------------------------
constexpr int kCombineThreads = 224;                        // 1792 float4 per row = 224 x 8
constexpr int kCombineRowVec = kHidden / 4 / kCombineThreads;
static_assert(kCombineRowVec * kCombineThreads * 4 == kHidden, "combine row split");

// VEC float4 columns per thread: a CTA covers VEC/8 of a token row
// (gridDim.y = 8 / VEC).  Large batches use whole rows per CTA (fewer, fuller
// CTAs, 8 loads in flight per thread); small ones split rows for parallelism.
template <int VEC>
__global__ void __launch_bounds__(kCombineThreads)
combine_kernel(const float* __restrict__ down, const int32_t* __restrict__ inv_row,
               const float* __restrict__ topk_w, int T, __nv_bfloat16* __restrict__ out,
               float* __restrict__ out_f32, const int* __restrict__ front_sync, int front_ctas,
               int* __restrict__ err) {
  griddep_wait();
  griddep_launch_dependents();
  const int t = blockIdx.x;
  __shared__ int s_row[kTopK];
  __shared__ float s_w[kTopK];
  // After the fused front kernel the GEMMs do not wait for its completion, so
  // when no GEMM work depended on it (no local rows) the grid dependency does
  // not cover it either: wait for its gather count (bounded) before reading
  // the routing and row map it wrote.
  if (front_sync != nullptr && threadIdx.x == 0) {
    volatile int ab = 0;
    if (!wait_counter(front_sync + 1, front_ctas, &ab)) raise_error(err, kDevTimeoutBarrier);
  }
  __syncthreads();
  __shared__ int s_n;
  if (threadIdx.x < 32) {   // this token's local picks, compacted in ascending k
    const int k = threadIdx.x;
    const int r = k < kTopK ? __ldcg(inv_row + (size_t)t * kTopK + k) : -1;
    const float wk = k < kTopK ? __ldcg(topk_w + (size_t)t * kTopK + k) : 0.f;
    const uint32_t m = __ballot_sync(0xffffffffu, r >= 0);
    if (r >= 0) {
      const int pos = __popc(m & ((1u << k) - 1u));
      s_row[pos] = r;
      s_w[pos] = wk;
    }
    if (k == 0) s_n = __popc(m);
  }
  __syncthreads();
  // Each thread owns VEC float4 columns and issues all of a pick's loads
  // before adding them (fp32 multiply-then-add in ascending k, as index_add_).
  const int n = s_n;
  const int v0 = blockIdx.y * VEC * kCombineThreads + threadIdx.x;
  float4 acc[VEC];
#pragma unroll
  for (int c = 0; c < VEC; ++c) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = 0; k < n; ++k) {
    const float w = s_w[k];
    const float4* src = reinterpret_cast<const float4*>(down + (size_t)s_row[k] * kHidden);
    float4 o[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) o[c] = __ldcs(src + v0 + c * kCombineThreads);
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
      acc[c].x = __fadd_rn(acc[c].x, __fmul_rn(o[c].x, w));
      acc[c].y = __fadd_rn(acc[c].y, __fmul_rn(o[c].y, w));
      acc[c].z = __fadd_rn(acc[c].z, __fmul_rn(o[c].z, w));
      acc[c].w = __fadd_rn(acc[c].w, __fmul_rn(o[c].w, w));
    }
  }
#pragma unroll
  for (int c = 0; c < VEC; ++c) {
    const int v = v0 + c * kCombineThreads;
    if (out_f32) {
      reinterpret_cast<float4*>(out_f32 + (size_t)t * kHidden)[v] = acc[c];
    } else {
      __nv_bfloat162 lo = __floats2bfloat162_rn(acc[c].x, acc[c].y);
      __nv_bfloat162 hi = __floats2bfloat162_rn(acc[c].z, acc[c].w);
      uint2 packed;
      packed.x = *reinterpret_cast<uint32_t*>(&lo);
      packed.y = *reinterpret_cast<uint32_t*>(&hi);
      reinterpret_cast<uint2*>(out + (size_t)t * kHidden)[v] = packed;
    }
  }
}

// --------------------------------------------------------------------------
// Launchers (programmatic dependent launch: each kernel may start while the
// previous one drains; griddepcontrol.wait orders its reads)
// --------------------------------------------------------------------------
cudaError_t launch_route(bool from_ids, const float* logits, const void* bias, int T,
                         float scaling, int local_offset, int E_l, int32_t* ids, float* w,
                         uint8_t* masks8, int NB8p, int* err, cudaStream_t st) {
  const int nb = (T + kRouteTokens - 1) / kRouteTokens;
  if (nb == 0) return cudaSuccess;
  const __nv_bfloat16* b = static_cast<const __nv_bfloat16*>(bias);
  if (from_ids)
    return launch_pdl(route_kernel<true>, dim3(nb), dim3(kRouteTokens * 32), 0, st, logits, b, T,
                      scaling, local_offset, E_l, ids, w, masks8, NB8p, err);
  return launch_pdl(route_kernel<false>, dim3(nb), dim3(kRouteTokens * 32), 0, st, logits, b, T,
                    scaling, local_offset, E_l, ids, w, masks8, NB8p, err);
}

cudaError_t launch_scan(const uint8_t* masks8, int NB8p, int32_t* bases, int NB, int E_l, int32_t* seg,
                        int bn1, int bn2, int4* tiles1, int4* tiles2, int32_t* sched,
                        int32_t* counters1, int nt1, int32_t* counters2, int nt2, int* ready,
                        cudaStream_t st) {
  return launch_pdl(scan_kernel, dim3(1), dim3(1024), 0, st, masks8, NB8p, bases, NB, E_l, seg, bn1, bn2,
                    tiles1, tiles2, sched, counters1, nt1, counters2, nt2, ready);
}

cudaError_t launch_scatter(const int32_t* ids, const uint8_t* masks8, int NB8p, const int32_t* bases, int T,
                           int E_l, int local_offset, int R_cap, const void* hidden,
                           const float* hs_scale, int32_t* inv_row, int32_t* row_token,
                           uint8_t* act, float* act_scale, cudaStream_t st) {
  const int nb = (T + kPermBlock - 1) / kPermBlock;
  if (nb == 0) return cudaSuccess;
  return launch_pdl(scatter_kernel, dim3(nb, kGatherChunks), dim3(kPermBlock * kTopK), 0, st, ids,
                    masks8, NB8p, bases, T, E_l, local_offset, R_cap, static_cast<const uint8_t*>(hidden),
                    hs_scale, inv_row, row_token, act, act_scale);
}

cudaError_t launch_front(const float* logits, const void* bias, int T, float scaling, int local_offset,
                         int E_l, int R_cap, int bn1, int bn2, int nt1, int nt2, const void* hidden,
                         const float* hs_scale, int32_t* ids, float* w, uint8_t* masks8, int NB8p,
                         int32_t* seg, int4* tiles1, int4* tiles2, int32_t* sched,
                         int32_t* counters1, int32_t* counters2, int* ready, int32_t* inv_row,
                         int32_t* row_token, uint8_t* act, float* act_scale, int* err, int* front_sync,
                         cudaStream_t st) {
  const int nb = (T + kRouteTokens - 1) / kRouteTokens;
  if (nb == 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nb);
  cfg.blockDim = dim3(kRouteTokens * 32);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int na = 1;
  if (nb > 1 && nb <= 8) {   // one cluster: hardware barrier instead of global atomics
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = nb;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    na = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, front_kernel, logits, static_cast<const __nv_bfloat16*>(bias), T, scaling,
                            local_offset, E_l, R_cap, bn1, bn2, nt1, nt2, static_cast<const uint8_t*>(hidden),
                            hs_scale, ids, w, masks8, NB8p, seg, tiles1, tiles2, sched, counters1, counters2, ready,
                            inv_row, row_token, act, act_scale, err, front_sync);
}

cudaError_t launch_combine(const float* down, const int32_t* inv_row, const float* w, int T,
                           void* out, float* out_f32, const int* front_sync, int* err, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  const int front_ctas = (T + kRouteTokens - 1) / kRouteTokens;
  if (T >= 512)
    return launch_pdl(combine_kernel<kCombineRowVec>, dim3(T, 1), dim3(kCombineThreads), 0, st, down, inv_row,
                      w, T, static_cast<__nv_bfloat16*>(out), out_f32, front_sync, front_ctas, err);
  return launch_pdl(combine_kernel<1>, dim3(T, kCombineRowVec), dim3(kCombineThreads), 0, st, down, inv_row, w,
                    T, static_cast<__nv_bfloat16*>(out), out_f32, front_sync, front_ctas, err);
}

}  // namespace moe

