// Grouped f16-operand GEMMs on CTA pairs (tcgen05 cta_group::2), for large
// batches.
//
// Same operands and numerics as gemm_f16.cu (weights converted e4m3 -> f16 in
// shared memory with their block scale, tokens in f16 with their scales
// applied, whole-K fp32 accumulation in TMEM), but each MMA is M = 256 over
// the two CTAs of a cluster: each CTA holds 128 weight rows (its half of A)
// and half of the token tile (its half of B), and receives its 128 rows x N
// accumulator in its own TMEM.  Per SM and per 64-wide K step this halves the
// token bytes (N/2 rows instead of N) for the same tensor work, and lets N
// reach 256 with two accumulators per CTA (the epilogue overlaps the next tile).
//
// GEMM1 (KIND 1): a pair covers 128 features; CTA c holds the X1 rows of
// features 64c..64c+63 (A rows 0-63) and their X2 rows (A rows 64-127), so its
// TMEM lanes 0-63 hold X1 and 64-127 X2 of the same features and SwiGLU pairs
// them through shared memory inside the CTA.
// GEMM2 (KIND 2): a pair covers 256 output rows, 128 per CTA.
//
// The leader CTA (rank 0) issues the MMAs.  Both CTAs load their halves by TMA
// and convert their weights; the peer's converters and epilogue arrive on the
// leader's barriers remotely, and the leader's tcgen05.commit arrives on the
// barriers of both CTAs (one commit per CTA).  Every wait is bounded.
//
// Warp roles per CTA: 0 TMA producer, 1 TMEM owner (+ MMA issuer on the
// leader), 2..9 weight converters, 10..13 epilogue.
//
// Status: correct (the stage tests run it under path override 3) but measured
// 2.3-3.8x slower than gemm_f16.cu on B200: each pipeline step takes ~1.2 us
// whatever the box sizes, ring depths, MMAs or conversions (diagnostic builds
// removed each in turn), the TMA loads of a step landing 3-4.5 us after issue
// and the peer CTA's a microsecond after the leader's.  It is not selected
// automatically.
#include "kernels.cuh"

#ifndef MOE_PAIR_RS
#define MOE_PAIR_RS 6
#define MOE_PAIR_OS 3
#endif
#ifndef MOE_PAIR_NCONV
#define MOE_PAIR_NCONV 8
#endif

namespace moe {

#ifdef MOE_PAIR_TL
// Diagnostics builds only: %globaltimer stamps of the first 256 pipeline
// steps of cluster 0, [cta][event][step].
__device__ unsigned long long g_pair_tl[2][6][256];
#define PAIR_TL(ev, i) do { if (blockIdx.x < 2 && (i) < 256) g_pair_tl[crank][ev][i] = globaltimer_ns(); } while (0)
#else
#define PAIR_TL(ev, i) ((void)0)
#endif

namespace pair {

constexpr float kAccUnscale = 1.0f / 256.0f;   // weights are converted as q * s * 2^8

__device__ __forceinline__ void convert16(uint4 src, float scale, uint4& lo, uint4& hi) {
  const uint32_t w[4] = {src.x, src.y, src.z, src.w};
  const __half2 s2 = __float2half2_rn(scale * 256.0f);
  uint32_t out[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __nv_fp8x2_storage_t pr = static_cast<__nv_fp8x2_storage_t>((w[i] >> (16 * h)) & 0xFFFF);
      __half2 v = __hmul2(__half2(__nv_cvt_fp8x2_to_halfraw2(pr, __NV_E4M3)), s2);
      out[i * 2 + h] = *reinterpret_cast<uint32_t*>(&v);
    }
  }
  lo = make_uint4(out[0], out[1], out[2], out[3]);
  hi = make_uint4(out[4], out[5], out[6], out[7]);
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_peer(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void arrive_cluster(uint32_t bar) {   // any CTA's barrier
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool test_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with acquire at cluster scope.  REMOTE: the phase is completed
// by the peer CTA (a remote arrive or a commit from the leader); such waits
// poll with the non-suspending test_wait, because a thread suspended in
// try_wait was measured to resume only after about a microsecond when the
// completing arrive comes from the other CTA.
template <bool REMOTE>
__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  auto poll = [&]() { return REMOTE ? test_wait_cluster(bar, parity) : try_wait_cluster(bar, parity); };
  if (poll()) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    if (poll()) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) { *abort_flag = 1; return false; }
  }
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc2(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// One arrive on the barrier at shared::cluster address `bar` (this CTA's or
// the peer's) once the MMAs this thread issued have completed.
__device__ __forceinline__ void commit2(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void mma2_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// kind::f16 instruction descriptor: A = B = f16, D = f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

}  // namespace pair

template <int KIND>
struct PairCfg {
  static constexpr int K = KIND == 1 ? kHidden : kInter;
  static constexpr int ATOMS = K / 64;                    // 64-wide K steps per tile
  static constexpr int NT = KIND == 1 ? kInter / 128 : kHidden / 256;   // units per token tile
  static constexpr int W_ROWS = KIND == 1 ? kGemm1Out : kHidden;
  static constexpr int BN = 256;                          // tokens per tile (pair N)
  static constexpr int HB = BN / 2;                       // token rows held by one CTA
  static constexpr int W8 = 128 * 64;                     // e4m3 weights: 128 rows x 64 B
  static constexpr int W16 = 128 * 128;                   // f16 weights, 128-byte swizzled
  static constexpr int RAW = W8 + HB * 128;               // raw stage: weights + token half
  static constexpr int RS = MOE_PAIR_RS, OS = MOE_PAIR_OS;
  static constexpr int OFF_OP = RS * RAW;
  static constexpr int OFF_AUX = OFF_OP + OS * W16;
  static constexpr int XBUF = 16 * 64 * 4;                // GEMM1: one chunk of silu(X2) [16][64]
  static constexpr int SMEM = 1024 + OFF_AUX + 1024 + XBUF;
  static constexpr int NCONV = MOE_PAIR_NCONV;
  static constexpr int CROWS = 128 / NCONV;
  static constexpr int EPI0 = 64 + 32 * NCONV;
  static constexpr int THREADS = EPI0 + 128;
  static constexpr int TMEM_COLS = 512;                   // two accumulators of BN columns
  static_assert(RAW % 1024 == 0 && W16 % 1024 == 0, "aligned stages");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

template <int KIND>
__global__ void __launch_bounds__(PairCfg<KIND>::THREADS, 1)
moe_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_b,
                     const GemmParams p) {
  using C = PairCfg<KIND>;
  using namespace pair;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* aux = smem + C::OFF_AUX;
  uint64_t* full = reinterpret_cast<uint64_t*>(aux);      // TMA bytes of raw stage s landed (local)
  uint64_t* empty = full + C::RS;                          // MMAs done with raw stage s (leader commit)
  uint64_t* conv = empty + C::RS;                          // leader: both CTAs converted stage o
  uint64_t* opempty = conv + C::OS;                        // MMAs done with operand stage o
  uint64_t* accf = opempty + C::OS;                        // accumulator b complete
  uint64_t* acce = accf + 2;                               // leader: both epilogues drained b
  uint64_t* drain = acce + 2;                              // all MMAs complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* last_flag = const_cast<int*>(abort_flag) + 1;
  float* xbuf = reinterpret_cast<float*>(aux + 1024);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_rank();
  const uint32_t peer = crank ^ 1u;
  const bool leader = crank == 0;

  griddep_wait();
  griddep_launch_dependents();
  const WorkSched sch = make_work_sched_for(p.sched[KIND - 1], C::NT, C::ATOMS, (int)gridDim.x / 2,
                                            (int)blockIdx.x / 2);
  const int n_iter = sch.n_iter();   // the same in both CTAs of the pair
  if (n_iter == 0) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::RS; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int o = 0; o < C::OS; ++o) { mbar_init(&conv[o], 2 * C::NCONV); mbar_init(&opempty[o], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&accf[b], 1); mbar_init(&acce[b], 8); }
    mbar_init(drain, 1);
    *const_cast<int*>(abort_flag) = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&tm_w); tma_prefetch_desc(&tm_b); }
  if (warp == 1) tmem_alloc2(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  cluster_sync();   // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (elect_one_lane()) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_b = l2_policy_evict_last();
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < n_iter; ++i) {
        int u, a, r;
        sch.at(i, C::ATOMS, u, a, r);
        const int2 mn = unit_tile(u, sch.n_mt, C::NT);
        const int4 tile = p.tiles[mn.x];
        const int s = i % C::RS;
        const bool got_empty = leader ? wait_bounded<false>(&empty[s], ((i / C::RS) & 1) ^ 1, abort_flag)
                                      : wait_bounded<true>(&empty[s], ((i / C::RS) & 1) ^ 1, abort_flag);
        if (!got_empty) { ok = false; break; }
        PAIR_TL(0, i);
        mbar_arrive_expect_tx(&full[s], C::W8 + p.box_rows * 128);
        uint8_t* st = smem + s * C::RAW;
        if (KIND == 1) {   // X1 rows then X2 rows of this CTA's 64 features
          const int f0 = tile.x * C::W_ROWS + mn.y * 128 + (int)crank * 64;
          tma_load_3d(&tm_w, &full[s], st, 0, a, f0, pol_w);
          tma_load_3d(&tm_w, &full[s], st + 64 * 64, 0, a, f0 + kInter, pol_w);
        } else {
          tma_load_3d(&tm_w, &full[s], st, 0, a, tile.x * C::W_ROWS + mn.y * 256 + (int)crank * 128, pol_w);
        }
        // this CTA's half of the token tile: rows [crank*N/2, (crank+1)*N/2) of N
        const int n_half = ((min(C::BN, (tile.z + 15) & ~15)) >> 1);
        tma_load_3d(&tm_b, &full[s], st + C::W8, 0, a, tile.y + (int)crank * n_half, pol_b);
        ++issued;
      }
      if (!ok) {
        raise_error(p.err, kDevTimeoutProducer);
        for (int i = max(0, issued - C::RS); i < issued; ++i) {
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[i % C::RS], (i / C::RS) & 1) && globaltimer_ns() - t0 < kWaitLimitNs / 10) {}
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    if (leader && elect_one_lane()) {
      const uint32_t smem_base = smem_u32(smem);
      auto both = [&](uint64_t* bar) {   // commit to this CTA's barrier and to the peer's
        commit2(smem_u32(bar));
        commit2(map_peer(smem_u32(bar), peer));
      };
      uint32_t idesc = 0;
      bool ok = true;
      int seg = 0;
      for (int i = 0; i < n_iter && ok; ++i) {
        int u, a, r;
        sch.at(i, C::ATOMS, u, a, r);
        const bool seg_first = (i == sch.n1) || (a == 0);
        const bool seg_last = (a == C::ATOMS - 1) || (i == n_iter - 1);
        const int b = seg & 1;
        if (seg_first) {
          const int rows = p.tiles[unit_tile(u, sch.n_mt, C::NT).x].z;
          idesc = idesc_f16(256, min(C::BN, (rows + 15) & ~15));
          if (!wait_bounded<true>(&acce[b], ((seg >> 1) & 1) ^ 1, abort_flag)) { ok = false; break; }
        }
        const int s = i % C::RS, o = i % C::OS;
        if (!wait_bounded<true>(&conv[o], (i / C::OS) & 1, abort_flag)) { ok = false; break; }
        PAIR_TL(4, i);
        tc_fence_after();
        const uint64_t adesc = make_sdesc_sw128(smem_base + C::OFF_OP + o * C::W16);
        const uint64_t bdesc = make_sdesc_sw128(smem_base + s * C::RAW + C::W8);
        const uint32_t d = tmem_base + (uint32_t)(b * C::BN);
#pragma unroll
        for (int k = 0; k < 4; ++k)   // 4 x K=16 per 128-byte atom; +32 B = +2 in addr>>4
          mma2_f16(d, adesc + 2 * k, bdesc + 2 * k, idesc, (seg_first && k == 0) ? 0u : 1u);
        both(&empty[s]);
        both(&opempty[o]);
        PAIR_TL(5, i);
        if (seg_last) { both(&accf[b]); ++seg; }
      }
      if (!ok) raise_error(p.err, kDevTimeoutMma);
      both(drain);
    }
    // Both CTAs: every MMA writing this CTA's TMEM has completed before teardown.
    if (elect_one_lane()) {
      const unsigned long long t0 = globaltimer_ns();
      while (!test_wait_cluster(drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {}
    }
    __syncwarp();
  } else if (warp < 2 + C::NCONV) {
    // ------------------------------------------------------------ weight converters (both CTAs)
    const int q = warp - 2;
    const uint32_t conv_bar0 = leader ? smem_u32(conv) : map_peer(smem_u32(conv), 0);
    for (int i = 0; i < n_iter; ++i) {
      int u, a, r;
      sch.at(i, C::ATOMS, u, a, r);
      const int2 mn = unit_tile(u, sch.n_mt, C::NT);
      const int e = p.tiles[mn.x].x;
      const int s = i % C::RS, o = i % C::OS;
      // block scale of this warp's rows: GEMM1 rows 0-63 are X1 (block nt),
      // 64-127 X2 (block 16+nt); GEMM2 rows are block 2*nt + crank
      const int nb = KIND == 1 ? mn.y + (q * C::CROWS >= 64 ? kInter / 128 : 0) : 2 * mn.y + (int)crank;
      const float wsc = __ldg(p.w_scale + ((size_t)e * (C::W_ROWS / 128) + nb) * (C::K / 128) + a / 2);
      if (!wait_bounded<false>(&full[s], (i / C::RS) & 1, abort_flag)) break;
      if (q == 0 && lane == 0) PAIR_TL(1, i);
      const bool got_op = leader ? wait_bounded<false>(&opempty[o], ((i / C::OS) & 1) ^ 1, abort_flag)
                                 : wait_bounded<true>(&opempty[o], ((i / C::OS) & 1) ^ 1, abort_flag);
      if (!got_op) break;
      if (q == 0 && lane == 0) PAIR_TL(2, i);
      const uint8_t* st = smem + s * C::RAW;
      uint8_t* opst = smem + C::OFF_OP + o * C::W16;
      const int part = lane & 3;
      uint4 src[C::CROWS / 8];
#pragma unroll
      for (int rr = 0; rr < C::CROWS / 8; ++rr) {
        const int row = q * C::CROWS + rr * 8 + (lane >> 2);
        src[rr] = *reinterpret_cast<const uint4*>(st + row * 64 + part * 16);
      }
#pragma unroll
      for (int rr = 0; rr < C::CROWS / 8; ++rr) {
        const int row = q * C::CROWS + rr * 8 + (lane >> 2);
        uint4 lo, hi;
        convert16(src[rr], wsc, lo, hi);
        uint8_t* dst = opst + row * 128;
        *reinterpret_cast<uint4*>(dst + (((2 * part) ^ (row & 7)) * 16)) = lo;
        *reinterpret_cast<uint4*>(dst + (((2 * part + 1) ^ (row & 7)) * 16)) = hi;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) arrive_cluster(conv_bar0 + (uint32_t)(o * sizeof(uint64_t)));
      if (q == 0 && lane == 0) PAIR_TL(3, i);
    }
    if (*abort_flag) raise_error(p.err, kDevTimeoutProducer);
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int et = threadIdx.x - C::EPI0;        // 0..127
    const int qq = warp & 3;                     // TMEM lane quarter
    const int f = qq * 32 + lane;                // accumulator row (TMEM lane)
    const uint32_t lane_addr = (uint32_t)(qq * 32) << 16;
    const uint32_t acce_bar0 = leader ? smem_u32(acce) : map_peer(smem_u32(acce), 0);
    int seg = 0, seg_a0 = 0;
    for (int i = 0; i < n_iter; ++i) {
      int u, a, r;
      sch.at(i, C::ATOMS, u, a, r);
      if (i == sch.n1 || a == 0) seg_a0 = a;
      const bool seg_last = (a == C::ATOMS - 1) || (i == n_iter - 1);
      if (!seg_last) continue;
      const int2 mn = unit_tile(u, sch.n_mt, C::NT);
      const int nt = mn.y;
      const int4 tile = p.tiles[mn.x];
      const int b = seg & 1;
      const bool got = leader ? wait_bounded<false>(&accf[b], (seg >> 1) & 1, abort_flag)
                              : wait_bounded<true>(&accf[b], (seg >> 1) & 1, abort_flag);
      if (named_bar_or(1, 128, !got || *abort_flag != 0)) break;
      tc_fence_after();
      const uint32_t acc0 = tmem_base + lane_addr + (uint32_t)(b * C::BN);
      const bool full_tile = (seg_a0 == 0 && a == C::ATOMS - 1);
      bool finish = true;
      int c_lo = 0, c_hi = -1;
      if (!full_tile) {
        // publish this CTA's rows of the share: [cta][slot][column][128 rows] fp32
        const int slot = sch.slot(sch.gid, r, C::ATOMS);
        float* mine = p.partials + ((size_t)blockIdx.x * 2 + slot) * C::BN * 128;
#pragma unroll 1
        for (int c0 = 0; c0 < tile.z; c0 += 16) {
          float v[16];
          tmem_ld16(acc0 + c0, v);
          tmem_ld_wait();
#pragma unroll
          for (int x = 0; x < 16; ++x) __stcg(mine + ((size_t)c0 + x) * 128 + f, v[x]);
        }
        __threadfence();
        c_lo = sch.first_cta(r, C::ATOMS);
        c_hi = sch.last_cta(r, C::ATOMS);
        named_bar_sync(1, 128);
        if (et == 0) {
          const int old = atomicAdd(p.counters + u * 2 + (int)crank, 1);
          last_flag[0] = (old == c_hi - c_lo) ? 1 : 0;
        }
        named_bar_sync(1, 128);
        finish = last_flag[0] != 0;
        if (finish) __threadfence();
      }
      if (finish) {
#pragma unroll 1
        for (int c0 = 0; c0 < tile.z; c0 += 16) {
          float v[16];
          if (full_tile) {
            tmem_ld16(acc0 + c0, v);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int x = 0; x < 16; ++x) v[x] = 0.f;
            for (int c = c_lo; c <= c_hi; ++c) {   // contributing pairs, fixed order
              const int cslot = sch.slot(c, r, C::ATOMS);
              const float* src = p.partials + ((size_t)(c * 2 + (int)crank) * 2 + cslot) * C::BN * 128;
#pragma unroll
              for (int x = 0; x < 16; ++x) v[x] += __ldcg(src + ((size_t)c0 + x) * 128 + f);
            }
          }
          if (KIND == 1) {
            // lanes 64-127 hold X2: silu(X2) to shared memory; lanes 0-63 (X1) finish
            if (f >= 64) {
#pragma unroll
              for (int x = 0; x < 16; ++x) {
                const float x2 = v[x] * kAccUnscale;
                xbuf[x * 64 + (f - 64)] = x2 * __frcp_rn(1.0f + __expf(-x2));
              }
            }
            named_bar_sync(1, 128);
            if (f < 64) {
#pragma unroll
              for (int x = 0; x < 16; ++x) {
                const int j = c0 + x;
                if (j >= tile.z) break;
                const float cv = v[x] * kAccUnscale * xbuf[x * 64 + f];
                p.inter16[(size_t)(tile.y + j) * kInter + nt * 128 + (int)crank * 64 + f] = __float2half_rn(cv);
              }
            }
            named_bar_sync(1, 128);
          } else {
#pragma unroll
            for (int x = 0; x < 16; ++x) {
              const int j = c0 + x;
              if (j >= tile.z) break;
              p.down[(size_t)(tile.y + j) * kHidden + nt * 256 + (int)crank * 128 + f] = v[x] * kAccUnscale;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_cluster(acce_bar0 + (uint32_t)(b * sizeof(uint64_t)));
      ++seg;
    }
    if (*abort_flag) raise_error(p.err, kDevTimeoutEpilogue);
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();   // no remote arrive or MMA touches this CTA after this point
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, C::TMEM_COLS);
  }
}

// --------------------------------------------------------------------------
template <int KIND>
static cudaError_t launch_pair_one(const CUtensorMap* tm_w, const CUtensorMap* tm_b, const GemmParams& p,
                                   int grid, cudaStream_t st) {
  using C = PairCfg<KIND>;
  auto kern = moe_gemm_pair_kernel<KIND>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, *tm_w, *tm_b, p);
}

int gemm_pair_grid(int kind, int sm_count) {
  // one cluster of two CTAs per SM pair, as many as can be resident at once
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count & ~1);
  cfg.blockDim = dim3(kind == 1 ? PairCfg<1>::THREADS : PairCfg<2>::THREADS);
  cfg.dynamicSmemBytes = kind == 1 ? PairCfg<1>::SMEM : PairCfg<2>::SMEM;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  cudaError_t e;
  if (kind == 1) {
    e = cudaFuncSetAttribute(moe_gemm_pair_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, PairCfg<1>::SMEM);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n, moe_gemm_pair_kernel<1>, &cfg);
  } else {
    e = cudaFuncSetAttribute(moe_gemm_pair_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, PairCfg<2>::SMEM);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n, moe_gemm_pair_kernel<2>, &cfg);
  }
  if (e != cudaSuccess || n <= 0) return 0;
  return 2 * (n < sm_count / 2 ? n : sm_count / 2);
}

size_t gemm_pair_partials_bytes(int grid) {
  return (size_t)grid * 2 * PairCfg<1>::BN * 128 * sizeof(float);
}

cudaError_t launch_gemm_pair(int kind, const CUtensorMap* tm_w, const CUtensorMap* tm_b, const GemmParams& p,
                             int grid, cudaStream_t st) {
  return kind == 1 ? launch_pair_one<1>(tm_w, tm_b, p, grid, st) : launch_pair_one<2>(tm_w, tm_b, p, grid, st);
}

}  // namespace moe

#ifdef MOE_PAIR_TL
extern "C" __attribute__((visibility("default"))) int moe_probe_pair_timeline(unsigned long long* host) {
  return cudaMemcpyFromSymbol(host, moe::g_pair_tl, sizeof(moe::g_pair_tl)) == cudaSuccess ? 0 : 1;
}
#endif

