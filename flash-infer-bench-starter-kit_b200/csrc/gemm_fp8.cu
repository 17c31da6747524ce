// Grouped FP8 block-scaled GEMMs of the MoE layer on the sm_100a tensor cores.
//
// Replaces the reference's CUTLASS grouped GEMMs
// (solution/python/moe_grouped_gemm_fp8.cu:821-948 and 956-1075) and its
// separate SwiGLU + requantisation kernel (solution/python/kernel.cu:1086-1145).
//
// Formulation ("swap AB"): the MMA's M=128 side is 128 weight rows, its N side
// is a tile of BN tokens, so a decode step with one token per expert still
// fills the tensor core's M dimension and the weight stream is the only large
// operand.  Both operands are K-major e4m3 tiles loaded by TMA with 128-byte
// swizzling; one tcgen05.mma of K=32 is issued four times per 128-wide K block.
// After the fused front kernel (small batches) the token operand of GEMM1 is
// gathered by the producer straight from hidden_states (tile::gather4, four
// 128-byte rows per copy, rows by the permuted-row -> token map); for larger
// batches it is the permuted activation the scatter kernel wrote, one TMA box
// per token tile, as is GEMM2's token operand (the intermediate).
//
// Block scales: the fp32 128x128 weight scale is a scalar per (tile, K block),
// the fp32 1x128 activation scale is per token column.  Because they are
// arbitrary fp32 values, each K block is accumulated into a fresh TMEM
// partial that the epilogue warps read (tcgen05.ld) and add into registers as
//     acc[j] += partial[j] * (w_scale * act_scale[j]).
// TMEM partials are double buffered so the MMA of block k+1 overlaps the
// promotion of block k.
//
// KIND 1 (GEMM1, 7168 -> 2x2048): each tile holds the X1 rows n..n+127 and the
// X2 rows 2048+n..2048+n+127 of W13, so SwiGLU c = silu(X2)*X1 and the 1x128
// requantisation of c are done in the epilogue.  c is stored as two e4m3
// terms, c ~= hi*s + lo*(s/16) with s = amax/448, written as the row pair
// (2r, 2r+1) of the intermediate.
// KIND 2 (GEMM2, 2048 -> 7168): the token operand holds the hi and lo rows of
// each token, so one MMA of N = 2*BN yields both; the epilogue folds them as
// (P_hi + P_lo/16) * s.
//
// K steps: one pipeline stage holds KS consecutive 128-wide K blocks, loaded
// by one 3D TMA box per operand ({128 bytes, rows, KS blocks}), because the
// TMA engine's cost is per box: fewer, larger boxes stream weights faster.
// Each K block still gets its own TMEM partial and its own scale promotion.
//
// Scheduling: persistent, one CTA per SM, stream-K.  The work is the list of
// (n-tile, token tile) units times K blocks; every CTA gets one contiguous
// range of that iteration space.  A unit split between CTAs is finished by the
// last contributor, which sums the partial tiles in fixed CTA order (so the
// result is deterministic) and runs the epilogue.
//
// Warp roles: warp 0 = TMA producer, warp 1 = TMEM owner + MMA issuer,
// warps 2.. = epilogue (one or two warpgroups, split by token columns).
#include "kernels.cuh"

namespace moe {

template <int KIND, int BN, int STAGES, int NWG, int KS, int OCC = 1>
struct GemmCfg {
  static constexpr int NW = KIND == 1 ? 2 : 1;              // weight tiles per K block
  static constexpr int MMA_N = KIND == 1 ? BN : 2 * BN;     // token-operand rows
  static constexpr int KB = KIND == 1 ? kHiddenBlocks : kInterBlocks;
  static constexpr int KSTEPS = KB / KS;                    // pipeline iterations per unit
  static constexpr int NT = KIND == 1 ? kInter / 128 : kHidden / 128;   // n-tiles per expert
  static constexpr int W_ROWS = KIND == 1 ? kGemm1Out : kHidden;        // weight rows per expert
  static constexpr int W_TILE = 128 * 128;
  static constexpr int B_TILE = MMA_N * 128;
  static constexpr int STAGE = KS * (NW * W_TILE + B_TILE);
  static constexpr int BUF_COLS = KS * NW * MMA_N;          // TMEM columns of one partial buffer
  static constexpr int NBUF = 4 * BUF_COLS <= 512 ? 4 : 2;
  static constexpr int TMEM_USED = NBUF * BUF_COLS;
  static constexpr int TMEM_COLS = TMEM_USED <= 32 ? 32 : TMEM_USED <= 64 ? 64
                                 : TMEM_USED <= 128 ? 128 : TMEM_USED <= 256 ? 256 : 512;
  static constexpr int NEPI = 128 * NWG;
  static constexpr int THREADS = 64 + NEPI;
  static constexpr int CPW = BN / NWG;                      // token columns per warpgroup
  static constexpr int SLOT = KS * NW * BN;                 // promotion coefficients per iteration
  static constexpr int RING = 3;                            // slots (prefetch distance 2)
  static constexpr int AUX = 2048 + RING * SLOT * 4 + NWG * 4 * CPW * 4 + (BN <= kGatherMaxBN ? BN * 4 : 0);
  static constexpr int SMEM = 1024 + STAGES * STAGE + AUX;
  static_assert(KB % KS == 0, "K steps");
  static_assert(TMEM_USED <= 512 && NBUF >= 2, "TMEM budget");
  static_assert(CPW % 16 == 0 || (KIND == 2 && CPW % 8 == 0), "column chunking");
  static_assert(MMA_N % 16 == 0 && MMA_N <= 256, "MMA N");
  static_assert(SLOT <= NEPI, "one coefficient per epilogue thread");
  static_assert(SMEM * OCC <= 228 * 1024 - OCC * 1024, "shared memory budget");
  static_assert(TMEM_COLS * OCC <= 512, "TMEM budget per SM");
};

template <int KIND, int BN, int STAGES, int NWG, int KS, int OCC>
__global__ void __launch_bounds__(GemmCfg<KIND, BN, STAGES, NWG, KS, OCC>::THREADS, OCC)
moe_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_b,
                const GemmParams p) {
  using C = GemmCfg<KIND, BN, STAGES, NWG, KS, OCC>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for 128-byte-swizzled TMA tiles.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* aux = smem + STAGES * C::STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(aux);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + C::NBUF;
  uint64_t* drain = tempty + C::NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* last_flag = const_cast<int*>(abort_flag) + 1;
  float* sring = reinterpret_cast<float*>(aux + 2048);     // [RING][SLOT] scales per iteration
  float* samax = sring + C::RING * C::SLOT;                // [NWG][4][CPW]
  int* s_tok = reinterpret_cast<int*>(samax + NWG * 4 * C::CPW);      // [BN] token of each tile row

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // GEMM1 waits for the routing/permutation kernels -- after the fused front
  // kernel only for its tile lists (front_sync[0]), so the weight stream starts
  // while the front kernel still gathers activations (front_sync[1] counts
  // gathered CTAs; activations and their scales are read after it completes).
  // GEMM2 does not wait for GEMM1 as a whole: it starts streaming its weights
  // on SMs GEMM1 has released and waits per expert (p.ready) before reading
  // the intermediate.
  const bool early1 = KIND == 1 && p.front_sync != nullptr;
  if (early1) {
    __shared__ int s_front_ok;
    if (threadIdx.x == 0) {
      volatile int ab = 0;
      s_front_ok = wait_counter(p.front_sync, 1, &ab) ? 1 : 0;
      if (!s_front_ok) raise_error(p.err, kDevTimeoutBarrier);
    }
    __syncthreads();
    if (!s_front_ok) return;   // uniform
  } else if (KIND == 1 || !p.early_start) {
    griddep_wait();
  }
  griddep_launch_dependents();
  const WorkSched sch = make_work_sched(p.sched[KIND - 1], C::NT, C::KSTEPS);
  const int n_iter = sch.n_iter();
  if (n_iter == 0) return;   // uniform: this CTA has no work

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < C::NBUF; ++b) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], NWG * 4); }
    mbar_init(drain, 1);
    *const_cast<int*>(abort_flag) = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&tm_w); tma_prefetch_desc(&tm_b); }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one_lane()) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_b = l2_policy_evict_last();
      int issued = 0;
      int ready_e = -1;                 // GEMM2: expert whose intermediate is known complete
      bool gathered = !early1;          // GEMM1 after the front kernel: row map and scales written
      [[maybe_unused]] int tok_mt = -1;   // token tile whose rows s_tok holds
      bool ok = true;
      for (int i = 0; i < n_iter; ++i) {
        int u, ks, r;
        sch.at(i, C::KSTEPS, u, ks, r);
        const int2 mn = unit_tile(u, sch.n_mt, C::NT);
        const int mt = mn.x, nt = mn.y;
        const int4 tile = p.tiles[mt];
        const int s = i % STAGES;
        if (!mbar_wait_bounded(&empty[s], ((i / STAGES) & 1) ^ 1, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(&full[s], C::STAGE);
        uint8_t* st = smem + s * C::STAGE;
        const int z = ks * KS;
        const int wrow = tile.x * C::W_ROWS + nt * 128;
        tma_load_3d(&tm_w, &full[s], st, 0, wrow, z, pol_w);
        if (KIND == 1) tma_load_3d(&tm_w, &full[s], st + KS * C::W_TILE, 0, wrow + kInter, z, pol_w);
        if (KIND == 2 && p.early_start && tile.x != ready_e) {
          const int cnt = p.seg[tile.x + 1] - p.seg[tile.x];
          const int target = (kInter / 128) * ((cnt + p.bn_prev - 1) / p.bn_prev);
          if (!wait_counter(p.ready + tile.x, target, abort_flag)) { ok = false; ++issued; break; }
          fence_proxy_async();
          ready_e = tile.x;
        }
        if (!gathered) {
          if (!wait_counter(p.front_sync + 1, p.front_ctas, abort_flag)) { ok = false; ++issued; break; }
          fence_proxy_async();
          gathered = true;
        }
        if constexpr (KIND == 1 && BN <= kGatherMaxBN) {
          if (p.row_token != nullptr) {
          // token rows straight from hidden_states: four rows per gather, rows
          // past the tile repeat its first token (their columns are not used)
          if (mt != tok_mt) {
            tok_mt = mt;
            for (int j = 0; j < BN; ++j) s_tok[j] = __ldcg(p.row_token + tile.y + (j < tile.z ? j : 0));
          }
          uint8_t* bdst = st + C::NW * KS * C::W_TILE;
          for (int kk = 0; kk < KS; ++kk)
            for (int g4 = 0; g4 < BN / 4; ++g4)
              tma_gather4(&tm_b, &full[s], bdst + kk * C::B_TILE + g4 * 512, (z + kk) * 128, s_tok[4 * g4],
                          s_tok[4 * g4 + 1], s_tok[4 * g4 + 2], s_tok[4 * g4 + 3], pol_b);
          } else {
            tma_load_3d(&tm_b, &full[s], st + C::NW * KS * C::W_TILE, 0, tile.y, z, pol_b);
          }
        } else {
          tma_load_3d(&tm_b, &full[s], st + C::NW * KS * C::W_TILE, 0, KIND == 1 ? tile.y : 2 * tile.y, z, pol_b);
        }
        ++issued;
      }
      if (!ok) {
        raise_error(p.err, kDevTimeoutProducer);
        // Let copies already in flight land before the CTA exits.
        for (int i = max(0, issued - STAGES); i < issued; ++i) {
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[i % STAGES], (i / STAGES) & 1) &&
                 globaltimer_ns() - t0 < kWaitLimitNs / 10) {}
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one_lane()) {
      const uint32_t smem_base = smem_u32(smem);
      bool ok = true;
      int cur_u = -1;
      uint32_t idesc = 0;
      for (int i = 0; i < n_iter; ++i) {
        const int s = i % STAGES, b = i % C::NBUF;
        const int u = sch.unit_of(i, C::KSTEPS);
        if (u != cur_u) {
          // MMA N covers the tile's rows only (KIND 2: hi and lo row per token).
          cur_u = u;
          const int rows = (KIND == 1 ? 1 : 2) * p.tiles[unit_tile(u, sch.n_mt, C::NT).x].z;
          idesc = make_idesc_f8(128, min(C::MMA_N, (rows + 15) & ~15));
        }
        if (!mbar_wait_bounded(&full[s], (i / STAGES) & 1, abort_flag)) { ok = false; break; }
        if (!mbar_wait_bounded(&tempty[b], ((i / C::NBUF) & 1) ^ 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t st = smem_base + s * C::STAGE;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          const uint64_t bdesc = make_sdesc_sw128(st + C::NW * KS * C::W_TILE + kk * C::B_TILE);
#pragma unroll
          for (int w = 0; w < C::NW; ++w) {
            const uint64_t adesc = make_sdesc_sw128(st + (w * KS + kk) * C::W_TILE);
            const uint32_t d = tmem_base + (uint32_t)(b * C::BUF_COLS + (kk * C::NW + w) * C::MMA_N);
#pragma unroll
            for (int k = 0; k < 4; ++k)   // 4 x K=32 per 128-byte K block; +32 B = +2 in addr>>4
              tc_mma_f8(d, adesc + 2 * k, bdesc + 2 * k, idesc, k > 0 ? 1u : 0u);
          }
        }
        tc_commit(&empty[s]);
        tc_commit(&tfull[b]);
      }
      if (!ok) raise_error(p.err, kDevTimeoutMma);
      // Wait for every MMA this thread issued before TMEM is released.
      tc_commit(drain);
      const unsigned long long t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {}
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int et = threadIdx.x - 64;            // 0 .. NEPI-1
    const int wg = et >> 7;                     // warpgroup -> token-column half
    const int q = warp & 3;                     // TMEM lane quarter this warp may access
    const int f = q * 32 + lane;                // weight row inside the 128-row tile
    const int j0 = wg * C::CPW;                 // first token column of this warpgroup
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;

    float acc[C::NW][C::CPW];
    int seg_k0 = 0;
    int4 tile = make_int4(0, 0, 0, 0);

    // Promotion coefficients of iteration i live in ring slot i % RING:
    // coef[kk][w][j] = weight-block scale (K block kk, weight tile w) x
    // token-column scale (K block kk, column j), 0 for columns past the tile.
    // Thread et < SLOT computes its entry two iterations ahead, so the loads
    // never sit on the critical path and the promotion is one FMA per element.
    const bool loader = et < C::SLOT;
    const int my_kk = et / (C::NW * BN), my_w = (et / BN) % C::NW, my_j = et % BN;
    int pf_unit = -1, pf_col = -1, pf_e = 0, pf_nt = 0;
    bool pf_gathered = !early1;
    auto fetch = [&](int i_t) -> float {
      int u_t, ks_t, r_t;
      sch.at(i_t, C::KSTEPS, u_t, ks_t, r_t);
      const int kb_t = ks_t * KS + my_kk;
      if (u_t != pf_unit) {
        pf_unit = u_t;
        const int2 mn = unit_tile(u_t, sch.n_mt, C::NT);
        const int4 tl = p.tiles[mn.x];
        pf_e = tl.x;
        pf_nt = mn.y;
        pf_col = my_j < tl.z ? tl.y + my_j : -1;
        if (KIND == 2 && p.early_start && pf_col >= 0) {   // the intermediate's scales come from GEMM1
          const int cnt = p.seg[pf_e + 1] - p.seg[pf_e];
          wait_counter(p.ready + pf_e, (kInter / 128) * ((cnt + p.bn_prev - 1) / p.bn_prev), abort_flag);
        }
      }
      if (pf_col < 0) return 0.f;
      if (!pf_gathered) {                               // act_scale is written by the front kernel
        wait_counter(p.front_sync + 1, p.front_ctas, abort_flag);
        pf_gathered = true;
      }
      const int nb = KIND == 1 ? pf_nt + my_w * (kInter / 128) : pf_nt;
      const float wsc = __ldg(p.w_scale + ((size_t)pf_e * (C::W_ROWS / 128) + nb) * C::KB + kb_t);
      const float* bs = p.b_scale + (size_t)kb_t * p.R_cap + pf_col;
      return wsc * (((KIND == 2 && p.early_start) || early1) ? __ldcg(bs) : __ldg(bs));
    };
    for (int i_t = 0; i_t < 2 && i_t < n_iter; ++i_t)
      if (loader) sring[i_t * C::SLOT + et] = fetch(i_t);
    named_bar_sync(1, C::NEPI);

    for (int i = 0; i < n_iter; ++i) {
      int u, ks, r;
      sch.at(i, C::KSTEPS, u, ks, r);
      const int2 mn = unit_tile(u, sch.n_mt, C::NT);
      const int mt = mn.x, nt = mn.y;
      const int b = i % C::NBUF;
      if (i == sch.n1 || ks == 0) {
        tile = p.tiles[mt];
        seg_k0 = ks;
#pragma unroll
        for (int w = 0; w < C::NW; ++w)
#pragma unroll
          for (int jj = 0; jj < C::CPW; ++jj) acc[w][jj] = 0.f;
      }
      const float pre = (loader && i + 2 < n_iter) ? fetch(i + 2) : 0.f;
      const float* sl = sring + (i % C::RING) * C::SLOT;
      const bool got = mbar_wait_warp(&tfull[b], (i / C::NBUF) & 1, abort_flag);
      if (got) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
          for (int w = 0; w < C::NW; ++w) {
            const float* coef = sl + (kk * C::NW + w) * BN + j0;
            const uint32_t col0 = (uint32_t)(b * C::BUF_COLS + (kk * C::NW + w) * C::MMA_N);
            // TMEM columns of this warpgroup: KIND 1 one per token, KIND 2 two
            // per token (hi, lo).  Loads of LDC columns, two in flight per wait.
            constexpr int TCOLS = KIND == 1 ? C::CPW : 2 * C::CPW;
            constexpr int LDC = 16;
            constexpr int NLD = TCOLS / LDC;
            const uint32_t tcol = col0 + (KIND == 1 ? j0 : 2 * j0);
#pragma unroll
            for (int c = 0; c < NLD; c += 2) {
              // Columns past the tile's rows hold no MMA result: skip them.
              if (j0 + c * (KIND == 1 ? LDC : LDC / 2) >= tile.z) break;
              float v[2][LDC];
              tmem_ld<LDC>(tmem_base + lane_addr + tcol + c * LDC, v[0]);
              if (c + 1 < NLD) tmem_ld<LDC>(tmem_base + lane_addr + tcol + (c + 1) * LDC, v[1]);
              tmem_ld_wait();
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                if (c + h >= NLD) break;
                constexpr int TOK = KIND == 1 ? LDC : LDC / 2;     // token columns per load
#pragma unroll
                for (int x4 = 0; x4 < TOK / 4; ++x4) {
                  const float4 cf = reinterpret_cast<const float4*>(coef + (c + h) * TOK)[x4];
                  const int jj = (c + h) * TOK + x4 * 4;
                  if (KIND == 1) {
                    const float* vv = v[h] + x4 * 4;
                    acc[w][jj + 0] = fmaf(vv[0], cf.x, acc[w][jj + 0]);
                    acc[w][jj + 1] = fmaf(vv[1], cf.y, acc[w][jj + 1]);
                    acc[w][jj + 2] = fmaf(vv[2], cf.z, acc[w][jj + 2]);
                    acc[w][jj + 3] = fmaf(vv[3], cf.w, acc[w][jj + 3]);
                  } else {
                    const float* vv = v[h] + x4 * 8;
                    acc[w][jj + 0] = fmaf(fmaf(vv[1], 0.0625f, vv[0]), cf.x, acc[w][jj + 0]);
                    acc[w][jj + 1] = fmaf(fmaf(vv[3], 0.0625f, vv[2]), cf.y, acc[w][jj + 1]);
                    acc[w][jj + 2] = fmaf(fmaf(vv[5], 0.0625f, vv[4]), cf.z, acc[w][jj + 2]);
                    acc[w][jj + 3] = fmaf(fmaf(vv[7], 0.0625f, vv[6]), cf.w, acc[w][jj + 3]);
                  }
                }
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
      }
      if (loader && i + 2 < n_iter) sring[((i + 2) % C::RING) * C::SLOT + et] = pre;
      if (named_bar_or(1, C::NEPI, *abort_flag != 0)) break;   // uniform abort decision

      const bool seg_last = (ks == C::KSTEPS - 1) || (i == n_iter - 1);
      if (!seg_last) continue;

      // ---------------- end of this CTA's share of unit u
      if (!(seg_k0 == 0 && ks == C::KSTEPS - 1)) {
        // stream-K: publish the partial, the last contributor finishes the unit
        const int slot = sch.slot(blockIdx.x, r, C::KSTEPS);
        float* mine = p.partials + ((size_t)(blockIdx.x * 2 + slot) * C::NW) * BN * 128;
#pragma unroll
        for (int w = 0; w < C::NW; ++w)
#pragma unroll
          for (int jj = 0; jj < C::CPW; ++jj)
            __stcg(mine + ((size_t)w * BN + j0 + jj) * 128 + f, acc[w][jj]);
        named_bar_sync(1, C::NEPI);
        const int c_lo = sch.first_cta(r, C::KSTEPS);
        const int c_hi = sch.last_cta(r, C::KSTEPS);
        if (et == 0) {
          const int old = atom_add_acq_rel_gpu(p.counters + u, 1);   // publishes this share, acquires the others
          last_flag[0] = (old == c_hi - c_lo) ? 1 : 0;
        }
        named_bar_sync(1, C::NEPI);
        if (!last_flag[0]) continue;
        if (c_hi - c_lo == 1) {
          // Two contributors: fp32 addition is commutative, so adding the other
          // CTA's partial to our registers is the same sum whoever is last.
          const int c = (c_lo == (int)blockIdx.x) ? c_hi : c_lo;
          const int cslot = sch.slot(c, r, C::KSTEPS);
          const float* src = p.partials + ((size_t)(c * 2 + cslot) * C::NW) * BN * 128;
          float other[C::NW][C::CPW];
#pragma unroll
          for (int w = 0; w < C::NW; ++w)
#pragma unroll
            for (int jj = 0; jj < C::CPW; ++jj)
              other[w][jj] = __ldcg(src + ((size_t)w * BN + j0 + jj) * 128 + f);
#pragma unroll
          for (int w = 0; w < C::NW; ++w)
#pragma unroll
            for (int jj = 0; jj < C::CPW; ++jj) acc[w][jj] += other[w][jj];
        } else {
          // Three or more: sum every published partial in ascending CTA order.
#pragma unroll
          for (int w = 0; w < C::NW; ++w)
#pragma unroll
            for (int jj = 0; jj < C::CPW; ++jj) acc[w][jj] = 0.f;
          for (int c = c_lo; c <= c_hi; ++c) {
            const int cslot = sch.slot(c, r, C::KSTEPS);
            const float* src = p.partials + ((size_t)(c * 2 + cslot) * C::NW) * BN * 128;
#pragma unroll
            for (int w = 0; w < C::NW; ++w)
#pragma unroll
              for (int jj = 0; jj < C::CPW; ++jj)
                acc[w][jj] += __ldcg(src + ((size_t)w * BN + j0 + jj) * 128 + f);
          }
        }
      }
      if (KIND == 1) {
        // SwiGLU: c = silu(X2) * X1, X1 = acc[0], X2 = acc[1]
        float* my_amax = samax + (wg * 4 + q) * C::CPW;
#pragma unroll
        for (int jj = 0; jj < C::CPW; ++jj) {
          const float x1 = acc[0][jj], x2 = acc[C::NW - 1][jj];
          const float cv = x2 * __frcp_rn(1.0f + __expf(-x2)) * x1;
          acc[0][jj] = cv;
          float m = fabsf(cv);
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
          if (lane == 0) my_amax[jj] = m;
        }
        named_bar_sync(2 + wg, 128);
#pragma unroll
        for (int jj = 0; jj < C::CPW; ++jj) {
          const float* am = samax + wg * 4 * C::CPW + jj;
          const float amax = fmaxf(fmaxf(am[0], am[C::CPW]), fmaxf(am[2 * C::CPW], am[3 * C::CPW]));
          const float s = amax > 0.f ? amax * (1.0f / kFp8Max) : 1.0f;
          const float inv = __frcp_rn(s);
          const float cv = acc[0][jj];
          const uint8_t hi = f32_to_e4m3(__fmul_rn(cv, inv));
          const float resid = __fsub_rn(cv, __fmul_rn(e4m3_to_f32(hi), s));
          const uint8_t lo = f32_to_e4m3(__fmul_rn(resid, __fmul_rn(inv, 16.0f)));
          const int j = j0 + jj;
          if (j < tile.z) {
            const size_t row = (size_t)(tile.y + j);
            p.inter[(2 * row) * kInter + nt * 128 + f] = hi;
            p.inter[(2 * row + 1) * kInter + nt * 128 + f] = lo;
            if (f == 0) p.inter_scale[(size_t)nt * p.R_cap + row] = s;
          }
        }
        if (p.early_start) {
          // all warpgroups' stores of this unit, then one release increment
          named_bar_sync(1, C::NEPI);
          if (et == 0) red_add_release_gpu(p.ready + tile.x, 1);
        } else {
          named_bar_sync(2 + wg, 128);
        }
      } else {
#pragma unroll
        for (int jj = 0; jj < C::CPW; ++jj) {
          const int j = j0 + jj;
          if (j < tile.z)
            p.down[(size_t)(tile.y + j) * kHidden + nt * 128 + f] = acc[0][jj];
        }
      }
    }
    if (*abort_flag) raise_error(p.err, kDevTimeoutEpilogue);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// --------------------------------------------------------------------------
// Host-side dispatch: (kind, BN) -> stages, warpgroups, K blocks per stage.
// --------------------------------------------------------------------------
template <int KIND, int BN> struct Pick;
template <> struct Pick<1, 16> { static constexpr int S = 3, W = 1, K = 2, O = 1; };
template <> struct Pick<1, 32> { static constexpr int S = 3, W = 1, K = 2, O = 1; };
template <> struct Pick<1, 64> { static constexpr int S = 2, W = 2, K = 2, O = 1; };
template <> struct Pick<1, 128> { static constexpr int S = 4, W = 2, K = 1, O = 1; };
template <> struct Pick<2, 16> { static constexpr int S = 2, W = 1, K = 4, O = 1; };
template <> struct Pick<2, 32> { static constexpr int S = 2, W = 1, K = 4, O = 1; };
template <> struct Pick<2, 64> { static constexpr int S = 3, W = 1, K = 2, O = 1; };
template <> struct Pick<2, 128> { static constexpr int S = 4, W = 2, K = 1, O = 1; };

template <int KIND, int BN>
using CfgOf = GemmCfg<KIND, BN, Pick<KIND, BN>::S, Pick<KIND, BN>::W, Pick<KIND, BN>::K, Pick<KIND, BN>::O>;

template <int KIND, int BN>
static cudaError_t launch_one(const CUtensorMap* tm_w, const CUtensorMap* tm_b, const GemmParams& p,
                              int grid, cudaStream_t st) {
  using P = Pick<KIND, BN>;
  using C = CfgOf<KIND, BN>;
  auto kern = moe_gemm_kernel<KIND, BN, P::S, P::W, P::K, P::O>;
  static std::atomic<void*> seen[kMaxCachedDevices];
  cudaError_t e = once_per_context(seen, [&] {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  });
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(grid), dim3(C::THREADS), C::SMEM, st, *tm_w, *tm_b, p);
}

#define MOE_GEMM_CASES(X) X(1, 16) X(1, 32) X(1, 64) X(1, 128) X(2, 16) X(2, 32) X(2, 64) X(2, 128)

size_t gemm_partials_bytes(int kind, int bn, int grid) {
#define X(KD, BB) \
  if (kind == KD && bn == BB) return (size_t)grid * 2 * CfgOf<KD, BB>::NW * BB * 128 * sizeof(float);
  MOE_GEMM_CASES(X)
#undef X
  return 0;
}

int gemm_k_per_stage(int kind, int bn) {
#define X(KD, BB) \
  if (kind == KD && bn == BB) return Pick<KD, BB>::K;
  MOE_GEMM_CASES(X)
#undef X
  return 0;
}

int gemm_ctas_per_sm(int kind, int bn) {
#define X(KD, BB) \
  if (kind == KD && bn == BB) return Pick<KD, BB>::O;
  MOE_GEMM_CASES(X)
#undef X
  return 1;
}

cudaError_t launch_gemm(int kind, int bn, const CUtensorMap* tm_w, const CUtensorMap* tm_b,
                        const GemmParams& p, int grid, cudaStream_t st) {
#define X(KD, BB) \
  if (kind == KD && bn == BB) return launch_one<KD, BB>(tm_w, tm_b, p, grid, st);
  MOE_GEMM_CASES(X)
#undef X
  return cudaErrorInvalidValue;
}

}  // namespace moe

