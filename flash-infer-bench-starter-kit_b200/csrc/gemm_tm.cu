// Grouped FP8 block-scaled GEMMs for large batches, tokens on the MMA's M side.
//
// Replaces, for prefill-sized batches, the reference's CUTLASS grouped GEMMs
// (solution/python/moe_grouped_gemm_fp8.cu:821-948 and 956-1075) and its
// SwiGLU + requantisation kernel (solution/python/kernel.cu:1086-1145).
//
// Orientation: the MMA's M = 128 side is a tile of up to 128 token rows of one
// expert, its N side is 128 weight rows (output features).  Each TMEM lane then
// holds one token row, so the block-scale promotion of a K block,
//     acc[j][f] += partial[j][f] * (act_scale[j][kb] * w_scale[nb][kb]),
// multiplies every column a thread owns by ONE scalar: no per-column
// coefficients, no shared-memory traffic, one FMA per element.  (The decode
// kernels in gemm_fp8.cu put weights on M instead, because a decode tile has a
// handful of tokens; there the coefficient varies per column.)
//
// GEMM1 (KIND 1, 7168 -> 2x2048): a unit is 128 tokens x 256 weight rows,
// half A = X1 rows n..n+127 of W13, half B = X2 rows 2048+n..; the epilogue
// forms c = silu(X2)*X1 and its 1x128 block scale per token, so SwiGLU and the
// requantisation never leave the SM.  c is stored as two e4m3 terms on the
// same scale s = amax/448, c ~= (hi + lo)*s, hi in plane 0 and lo in plane 1
// of the intermediate [2][R_cap][2048].
// GEMM2 (KIND 2, 2048 -> 7168): a unit is 128 tokens x 128 hidden rows; each
// K block runs two MMAs into the same partial, one with the hi plane and one
// with the lo plane (they share the scale s), so the two-term intermediate
// costs MMA time but no extra promotion.
//
// TMEM holds NSLOT K-block partials of a whole unit (GEMM1 2 x 256 columns,
// GEMM2 4 x 128), so the tensor core runs one (three) K blocks ahead of the
// epilogue warps promoting the oldest one.  The running accumulators live in
// registers: each of the 256 epilogue threads owns one token row (its TMEM
// lane) and 64 columns of each half (GEMM1: 128 fp32 values, hence two
// warpgroups and 168 registers per thread; a block of 10 warps leaves that
// many).
//
// Pipeline: TMA producer (warp 8) -> STAGES-deep ring of {token tile(s), two
// weight tiles, their block scales} per K step -> MMA issuer (warp 9, also
// owns TMEM) -> 2 epilogue warpgroups (warps 0..7; warp w reads TMEM lanes
// 32*(w%4)..).  Epilogue warpgroup g owns columns 64g..64g+63 of both halves,
// so the SwiGLU of a feature (X1 in half A, X2 in half B) stays in one
// thread; the per-token amax of a 128-feature block is combined through
// shared memory.
//
// Scheduling: the persistent wave + stream-K schedule of the other GEMM
// families (WorkSched); a unit split between CTAs publishes every share to
// global memory and its last contributor adds them in ascending CTA order, so
// the result is bitwise deterministic.
#include "kernels.cuh"

namespace moe {

template <int KIND, int KS, int STAGES>
struct TmCfg {
  static constexpr int K = KIND == 1 ? kHidden : kInter;
  static constexpr int KB = K / 128;                        // 128-wide K blocks
  static constexpr int KSTEPS = KB / KS;                    // pipeline iterations per unit
  // Output columns of a unit: NH halves of 128 (GEMM1: X1 and X2 of 128
  // features, so SwiGLU and the 1x128 requantisation stay in one unit; GEMM2:
  // 128 hidden rows).  TMEM holds NSLOT K-block partials of a whole unit.
  static constexpr int NH = KIND == 1 ? 2 : 1;
  static constexpr int NSLOT = 512 / (NH * 128);
  static constexpr int NT = KIND == 1 ? kInter / 128 : kHidden / 128;   // units per token tile
  static constexpr int W_ROWS = KIND == 1 ? kGemm1Out : kHidden;        // weight rows per expert
  static constexpr int NA = KIND == 1 ? 1 : 2;              // token tiles per K block (GEMM2: hi, lo)
  static constexpr int TILE = 128 * 128;                    // one [128 rows x 128 B] operand tile
  static constexpr int OFF_WA = KS * NA * TILE;             // weight tiles inside a stage
  static constexpr int OFF_WB = OFF_WA + KS * TILE;
  static constexpr int STAGE = OFF_WA + NH * KS * TILE;
  static constexpr int NEPI = 256;                          // two epilogue warpgroups (warps 0..7)
  static constexpr int W_PROD = 8, W_MMA = 9;               // producer and MMA warps
  static constexpr int THREADS = NEPI + 64;
  static constexpr int COLS = 64;                           // columns of each half per epilogue thread
  // Block scales travel in their own ring of SR slots, one per pipeline
  // iteration: KS rows of 132 fp32 token scales (a TMA box starting at the
  // tile's first row rounded down to a multiple of 4, so its x coordinate is
  // 16-byte aligned) and the two halves' weight scales (a box of 4 K blocks
  // per half, likewise aligned).  A separate, deeper ring lets an operand
  // stage be refilled as soon as its MMAs are done, however far the epilogue
  // lags behind the tensor core.
  static constexpr int SR = 8;
  static constexpr int SC_ROW = 132;
  static constexpr int SC_ACT = KS * SC_ROW * 4;
  static constexpr int SC_SLOT = ((SC_ACT + 127) / 128) * 128 + 128;
  static constexpr int SC_TX = SC_ACT + NH * 4 * 4;
  static constexpr int OFF_SC = 2048 + 2 * 2 * 128 * 4;    // after barriers + amax exchange [2][2][128]
  static constexpr int AUX = OFF_SC + SR * SC_SLOT;
  static constexpr int SMEM = 1024 + STAGES * STAGE + AUX;
  static_assert(KS == 1 || KS == 2 || KS == 4, "weight-scale boxes cover 4 aligned K blocks");
  static constexpr uint32_t SLOT_COLS = NH * 128, P_B = 128;   // partial slot: half A at +0, half B at +128
  static constexpr int PART_COLS = NH * 128;
  // GEMM1 with one K block per stage: both weight halves form one N = 256 operand
  static constexpr bool WIDE = KIND == 1 && KS == 1;
  static constexpr int PART_FLOATS = 128 * 256;             // one published share slot: [128 rows][<= 256 cols]
  static_assert(KB % KS == 0, "K steps");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

template <int KIND, int KS, int STAGES>
__global__ void __launch_bounds__(TmCfg<KIND, KS, STAGES>::THREADS, 1)
moe_gemm_tm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_b,
                   const __grid_constant__ CUtensorMap tm_bs, const __grid_constant__ CUtensorMap tm_ws,
                   const GemmParams p) {
  using C = TmCfg<KIND, KS, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* aux = smem + STAGES * C::STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(aux);        // TMA bytes of stage s landed
  uint64_t* empty = full + STAGES;                          // MMAs finished reading stage s
  uint64_t* pfull = empty + STAGES;                         // [NSLOT] partial slot written
  uint64_t* pempty = pfull + C::NSLOT;                      // [NSLOT] partial slot read
  uint64_t* sfull = pempty + C::NSLOT;                      // [SR] scales of an iteration landed
  uint64_t* sempty = sfull + C::SR;                         // [SR] scales read by every epilogue warp
  uint64_t* drain = sempty + C::SR;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* last_flag = const_cast<int*>(abort_flag) + 1;
  float* s_amax = reinterpret_cast<float*>(aux + 2048);     // [2 buffers][2 warpgroups][128 rows]
  uint8_t* s_sc = aux + C::OFF_SC;                          // [SR][SC_SLOT] scales per iteration

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  griddep_wait();
  griddep_launch_dependents();
  const WorkSched sch = make_work_sched(p.sched[KIND - 1], C::NT, C::KSTEPS);
  const int n_iter = sch.n_iter();
  if (n_iter == 0) return;   // uniform: this CTA has no work

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int s = 0; s < C::SR; ++s) { mbar_init(&sfull[s], 1); mbar_init(&sempty[s], C::NEPI / 32); }
    for (int h = 0; h < C::NSLOT; ++h) { mbar_init(&pfull[h], 1); mbar_init(&pempty[h], C::NEPI / 32); }
    mbar_init(drain, 1);
    *const_cast<int*>(abort_flag) = 0;
    fence_mbar_init();
  }
  if (warp == C::W_PROD && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_b);
    tma_prefetch_desc(&tm_bs);
    tma_prefetch_desc(&tm_ws);
  }
  if (warp == C::W_MMA) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == C::W_PROD) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one_lane()) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_b = l2_policy_evict_last();
      int issued = 0, sissued = 0;
      bool ok = true;
      for (int i = 0; i < n_iter; ++i) {
        int u, ks, r;
        sch.at(i, C::KSTEPS, u, ks, r);
        const int2 mn = unit_tile(u, sch.n_mt, C::NT);
        const int4 tile = p.tiles[mn.x];
        const int s = i % STAGES;
        if (!mbar_wait_bounded(&empty[s], ((i / STAGES) & 1) ^ 1, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(&full[s], C::STAGE);
        uint8_t* st = smem + s * C::STAGE;
        const int z = ks * KS;
        // Two operand boxes per stage (fewer, larger TMA boxes stream faster):
        // GEMM1 tokens {128 B, 128 rows, KS} + weights {128 B, 128 rows, KS,
        // X1|X2} (W13 viewed as [2E_l][56][2048][128 B]); GEMM2 tokens {128 B,
        // 128 rows, KS, hi|lo} + weights {128 B, 128 rows, KS}.
        if (KIND == 1) {
          tma_load_3d(&tm_b, &full[s], st, 0, tile.y, z, pol_b);
          tma_load_4d(&tm_w, &full[s], st + C::OFF_WA, 0, mn.y * 128, z, 2 * tile.x, pol_w);
        } else {
          tma_load_4d(&tm_b, &full[s], st, 0, tile.y, z, 0, pol_b);
          tma_load_3d(&tm_w, &full[s], st + C::OFF_WA, 0, tile.x * C::W_ROWS + mn.y * 128, z, pol_w);
        }
        ++issued;
        // this iteration's block scales into scale slot i % SR
        const int q = i % C::SR;
        if (!mbar_wait_bounded(&sempty[q], ((i / C::SR) & 1) ^ 1, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(&sfull[q], C::SC_TX);
        uint8_t* sc = s_sc + q * C::SC_SLOT;
        tma_load_2d(&tm_bs, &sfull[q], sc, tile.y & ~3, z, pol_b);
        if (KIND == 1)   // w_scale viewed as {56 K blocks, 16 n-blocks, 2 halves x E_l}
          tma_load_3d(&tm_ws, &sfull[q], sc + C::SC_SLOT - 128, z & ~3, mn.y, 2 * tile.x, pol_b);
        else             // w_scale viewed as {16 K blocks, 56 n-blocks, E_l}
          tma_load_3d(&tm_ws, &sfull[q], sc + C::SC_SLOT - 128, z & ~3, mn.y, tile.x, pol_b);
        ++sissued;
      }
      if (!ok) {
        raise_error(p.err, kDevTimeoutProducer);
        for (int i = max(0, issued - STAGES); i < issued; ++i) {   // let copies in flight land
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[i % STAGES], (i / STAGES) & 1) &&
                 globaltimer_ns() - t0 < kWaitLimitNs / 10) {}
        }
        for (int i = max(0, sissued - C::SR); i < sissued; ++i) {
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(&sfull[i % C::SR], (i / C::SR) & 1) &&
                 globaltimer_ns() - t0 < kWaitLimitNs / 10) {}
        }
      }
    }
  } else if (warp == C::W_MMA) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one_lane()) {
      const uint32_t smem_base = smem_u32(smem);
      constexpr uint32_t idesc = make_idesc_f8(128, 128);
      constexpr uint32_t idesc_wide = make_idesc_f8(128, 256);
      bool ok = true;
      int g = 0;                       // K blocks issued so far (slot g % NSLOT, phase (g / NSLOT) & 1)
      for (int i = 0; i < n_iter && ok; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait_bounded(&full[s], (i / STAGES) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t st = smem_base + s * C::STAGE;
#pragma unroll 1
        for (int kk = 0; kk < KS; ++kk, ++g) {
          const int slot = g % C::NSLOT;
          if (!mbar_wait_bounded(&pempty[slot], ((g / C::NSLOT) & 1) ^ 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          if (C::WIDE) {
            // GEMM1: the X1 and X2 weight tiles sit back to back (rows 0..255 of
            // one K-major operand), so one N = 256 MMA per K slice fills both
            // halves of the partial and the token tile is read once, not twice.
            const uint64_t adesc = make_sdesc_sw128(st + kk * C::TILE);
            const uint64_t bdesc = make_sdesc_sw128(st + C::OFF_WA);
            const uint32_t d = tmem_base + slot * C::SLOT_COLS;
#pragma unroll
            for (int k = 0; k < 4; ++k)   // 4 x K=32 per 128-byte K block; +32 B = +2 in addr>>4
              tc_mma_f8(d, adesc + 2 * k, bdesc + 2 * k, idesc_wide, k == 0 ? 0u : 1u);
          } else {
#pragma unroll
            for (int h = 0; h < C::NH; ++h) {
              const uint64_t bdesc = make_sdesc_sw128(st + (h ? C::OFF_WB : C::OFF_WA) + kk * C::TILE);
              const uint32_t d = tmem_base + slot * C::SLOT_COLS + (h ? C::P_B : 0u);
#pragma unroll
              for (int a = 0; a < C::NA; ++a) {
                const uint64_t adesc = make_sdesc_sw128(st + (a * KS + kk) * C::TILE);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                  tc_mma_f8(d, adesc + 2 * k, bdesc + 2 * k, idesc, (a == 0 && k == 0) ? 0u : 1u);
              }
            }
          }
          tc_commit(&pfull[slot]);
        }
        if (!ok) break;
        tc_commit(&empty[s]);
      }
      if (!ok) raise_error(p.err, kDevTimeoutMma);
      tc_commit(drain);
      const unsigned long long t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {}
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int et = threadIdx.x;                 // 0..255
    const int wg = et >> 7;                     // column group: columns 64wg..64wg+63 of each half
    const int q = warp & 3;                     // TMEM lane quarter of this warp
    const int j = q * 32 + lane;                // token row inside the tile (TMEM lane)
    const uint32_t lane_addr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(wg * C::COLS);
    const int col0 = wg * C::COLS;

    float acc[C::NH][C::COLS];                  // running sums: [half][column]
    int g = 0;                                  // K blocks consumed (slot g % NSLOT)
    int seg_k0 = 0;
    int nseg = 0;                               // segments finished (amax buffer parity)
    int4 tile = make_int4(0, 0, 0, 0);
    int nt = 0;
    bool row_ok = false;
    bool aborted = false;

    for (int i = 0; i < n_iter && !aborted; ++i) {
      int u, ks, r;
      sch.at(i, C::KSTEPS, u, ks, r);
      if (i == sch.n1 || ks == 0 || i == 0) {
        const int2 mn = unit_tile(u, sch.n_mt, C::NT);
        tile = p.tiles[mn.x];
        nt = mn.y;
        row_ok = j < tile.z;
        seg_k0 = ks;
#pragma unroll
        for (int h = 0; h < C::NH; ++h)
#pragma unroll
          for (int x = 0; x < C::COLS; ++x) acc[h][x] = 0.f;
      }
      // this iteration's scales: promotion coefficients of its K blocks
      const int sq = i % C::SR;
      float cA[KS], cB[KS];
      if (!mbar_wait_warp(&sfull[sq], (i / C::SR) & 1, abort_flag)) aborted = true;
      if (!aborted) {
        const float* sc = reinterpret_cast<const float*>(s_sc + sq * C::SC_SLOT);
        const float* wsc = reinterpret_cast<const float*>(s_sc + sq * C::SC_SLOT + C::SC_SLOT - 128);
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          const float as = row_ok ? sc[kk * C::SC_ROW + (tile.y & 3) + j] : 0.f;
          const int x = (ks * KS + kk) & 3;
          cA[kk] = as * wsc[x];
          cB[kk] = C::NH > 1 ? as * wsc[4 + x] : 0.f;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sempty[sq]);
      }
#pragma unroll
      for (int kk = 0; kk < KS && !aborted; ++kk, ++g) {
        const int slot = g % C::NSLOT;
        if (!mbar_wait_warp(&pfull[slot], (g / C::NSLOT) & 1, abort_flag)) { aborted = true; break; }
        tc_fence_after();
        const uint32_t pbase = lane_addr + slot * C::SLOT_COLS;
        // 4*NH chunks of 16 columns (4 per half), two loads in flight
#pragma unroll
        for (int cc = 0; cc < 4 * C::NH; cc += 2) {
          float pv[2][16];
          tmem_ld16(pbase + (cc >> 2) * C::P_B + (cc & 3) * 16, pv[0]);
          tmem_ld16(pbase + ((cc + 1) >> 2) * C::P_B + ((cc + 1) & 3) * 16, pv[1]);
          tmem_ld_wait();
          if (cc == 4 * C::NH - 2) {            // every load of this slot is done: release it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&pempty[slot]);
          }
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int h = (cc + e) >> 2, c0 = ((cc + e) & 3) * 16;
            const float cf = h ? cB[kk] : cA[kk];
            const float2 cf2 = make_float2(cf, cf);
#pragma unroll
            for (int x = 0; x < 16; x += 2) {   // paired FMAs (one fma.rn.f32x2 per two columns)
              const float2 r = __ffma2_rn(make_float2(pv[e][x], pv[e][x + 1]), cf2,
                                          make_float2(acc[h][c0 + x], acc[h][c0 + x + 1]));
              acc[h][c0 + x] = r.x;
              acc[h][c0 + x + 1] = r.y;
            }
          }
        }
      }
      const bool seg_last = (ks == C::KSTEPS - 1) || (i == n_iter - 1);
      if (!seg_last && !aborted) continue;
      // uniform abort decision at the end of each share (and on abort)
      if (named_bar_or(1, C::NEPI, aborted || *abort_flag != 0)) { aborted = true; break; }

      // ---------------- end of this CTA's share of unit u
      const bool full_unit = seg_k0 == 0 && ks == C::KSTEPS - 1;
      if (!full_unit) {
        // stream-K: publish this share, the last contributor adds all of them
        // in ascending CTA order (its own share included, re-read)
        float* mine = p.partials + (size_t)(blockIdx.x * 2 + sch.slot(blockIdx.x, r, C::KSTEPS)) * C::PART_FLOATS +
                      (size_t)j * C::PART_COLS + col0;
#pragma unroll
        for (int h = 0; h < C::NH; ++h)
#pragma unroll
          for (int w = 0; w < C::COLS / 4; ++w)
            __stcg(reinterpret_cast<float4*>(mine + h * 128) + w,
                   make_float4(acc[h][4 * w], acc[h][4 * w + 1], acc[h][4 * w + 2], acc[h][4 * w + 3]));
        named_bar_sync(1, C::NEPI);
        const int c_lo = sch.first_cta(r, C::KSTEPS);
        const int c_hi = sch.last_cta(r, C::KSTEPS);
        if (et == 0) {
          const int old = atom_add_acq_rel_gpu(p.counters + u, 1);   // publishes this share, acquires the others
          last_flag[0] = (old == c_hi - c_lo) ? 1 : 0;
        }
        named_bar_sync(1, C::NEPI);
        if (!last_flag[0]) continue;
#pragma unroll
        for (int h = 0; h < C::NH; ++h)
#pragma unroll
          for (int x = 0; x < C::COLS; ++x) acc[h][x] = 0.f;
        for (int c = c_lo; c <= c_hi; ++c) {
          const float* src = p.partials + (size_t)(c * 2 + sch.slot(c, r, C::KSTEPS)) * C::PART_FLOATS +
                             (size_t)j * C::PART_COLS + col0;
#pragma unroll
          for (int h = 0; h < C::NH; ++h)
#pragma unroll
            for (int w = 0; w < C::COLS / 4; ++w) {
              const float4 f = __ldcg(reinterpret_cast<const float4*>(src + h * 128) + w);
              acc[h][4 * w] += f.x;
              acc[h][4 * w + 1] += f.y;
              acc[h][4 * w + 2] += f.z;
              acc[h][4 * w + 3] += f.w;
            }
        }
      }
      const size_t row = (size_t)(tile.y + j);
      if (KIND == 1) {
        // SwiGLU c = silu(X2) * X1 (X1 = half A, X2 = half B), into acc[0]
        float m = 0.f;
#pragma unroll
        for (int x = 0; x < C::COLS; ++x) {
          const float x2 = acc[C::NH - 1][x];
          acc[0][x] = x2 * __frcp_rn(1.0f + __expf(-x2)) * acc[0][x];
          m = fmaxf(m, fabsf(acc[0][x]));
        }
        // 1x128 block scale over the 128 features of this unit, per token
        float* am = s_amax + (nseg & 1) * 2 * 128;
        am[wg * 128 + j] = m;
        named_bar_sync(1, C::NEPI);
        const float amax = fmaxf(am[j], am[128 + j]);
        const float sc = amax > 0.f ? amax * (1.0f / kFp8Max) : 1.0f;
        const float inv = __frcp_rn(sc);
#pragma unroll
        for (int ch = 0; ch < C::COLS / 16; ++ch) {
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            uint32_t hb = 0, lb = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const float cv = acc[0][16 * ch + 4 * w + b];
              const uint8_t hi = f32_to_e4m3(__fmul_rn(cv, inv));
              const float resid = __fsub_rn(cv, __fmul_rn(e4m3_to_f32(hi), sc));
              const uint8_t lo = f32_to_e4m3(__fmul_rn(resid, inv));
              hb |= (uint32_t)hi << (8 * b);
              lb |= (uint32_t)lo << (8 * b);
            }
            hw[w] = hb;
            lw[w] = lb;
          }
          if (row_ok) {
            *reinterpret_cast<uint4*>(p.inter + row * kInter + nt * 128 + col0 + 16 * ch) =
                make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4*>(p.inter + ((size_t)p.R_cap + row) * kInter + nt * 128 + col0 + 16 * ch) =
                make_uint4(lw[0], lw[1], lw[2], lw[3]);
          }
        }
        if (row_ok && wg == 0) p.inter_scale[(size_t)nt * p.R_cap + row] = sc;
      } else if (row_ok) {
#pragma unroll
        for (int h = 0; h < C::NH; ++h) {
          float4* d = reinterpret_cast<float4*>(p.down + row * kHidden + nt * (C::NH * 128) + h * 128 + col0);
#pragma unroll
          for (int w = 0; w < C::COLS / 4; ++w)
            d[w] = make_float4(acc[h][4 * w], acc[h][4 * w + 1], acc[h][4 * w + 2], acc[h][4 * w + 3]);
        }
      }
      ++nseg;
    }
    if (*abort_flag) raise_error(p.err, kDevTimeoutEpilogue);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == C::W_MMA) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// --------------------------------------------------------------------------
// Host-side dispatch
// --------------------------------------------------------------------------
template <int KIND> struct TmPick;   // K blocks per stage, stages
template <> struct TmPick<1> { static constexpr int KS = 1, S = 4; };
template <> struct TmPick<2> { static constexpr int KS = 1, S = 4; };

template <int KIND>
using TmCfgOf = TmCfg<KIND, TmPick<KIND>::KS, TmPick<KIND>::S>;

size_t gemm_tm_partials_bytes(int grid) {
  return (size_t)grid * 2 * TmCfgOf<1>::PART_FLOATS * sizeof(float);
}

int gemm_tm_k_per_stage(int kind) { return kind == 1 ? TmPick<1>::KS : TmPick<2>::KS; }

int gemm_tm_scale_box_cols() { return TmCfgOf<1>::SC_ROW; }

int gemm_tm_units_per_tile(int kind) { return kind == 1 ? TmCfgOf<1>::NT : TmCfgOf<2>::NT; }

template <int KIND>
static cudaError_t launch_tm_one(const CUtensorMap* tm_w, const CUtensorMap* tm_b, const CUtensorMap* tm_bs,
                                 const CUtensorMap* tm_ws, const GemmParams& p, int grid, cudaStream_t st) {
  using P = TmPick<KIND>;
  using C = TmCfgOf<KIND>;
  auto kern = moe_gemm_tm_kernel<KIND, P::KS, P::S>;
  static std::atomic<void*> seen[kMaxCachedDevices];
  cudaError_t e = once_per_context(seen, [&] {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  });
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(grid), dim3(C::THREADS), C::SMEM, st, *tm_w, *tm_b, *tm_bs, *tm_ws, p);
}

cudaError_t launch_gemm_tm(int kind, const CUtensorMap* tm_w, const CUtensorMap* tm_b, const CUtensorMap* tm_bs,
                           const CUtensorMap* tm_ws, const GemmParams& p, int grid, cudaStream_t st) {
  if (kind == 1) return launch_tm_one<1>(tm_w, tm_b, tm_bs, tm_ws, p, grid, st);
  if (kind == 2) return launch_tm_one<2>(tm_w, tm_b, tm_bs, tm_ws, p, grid, st);
  return cudaErrorInvalidValue;
}

}  // namespace moe
