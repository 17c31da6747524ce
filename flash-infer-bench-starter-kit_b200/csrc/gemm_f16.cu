// Grouped GEMMs for large batches (from 1536 tokens by default): block scales folded into
// f16 operands, whole-K accumulation in TMEM.
//
// The e4m3 GEMMs (gemm_fp8.cu) must promote every 128-wide K block from TMEM
// into registers because the fp32 block scales cannot enter an fp8 MMA.  For
// large token tiles that promotion costs more registers and issue slots than a
// CTA has.  Here the scales are applied to the operands instead:
//   * the token operand arrives in f16 with its 1x128 scales already applied
//     (the scatter kernel writes it that way for GEMM1; GEMM1's epilogue writes
//     the SwiGLU output in f16 for GEMM2);
//   * the weight tile is loaded in e4m3 by TMA and converted to f16 with its
//     128x128 block scale by four converter warps, straight into the 128-byte
//     swizzled K-major layout the MMA reads;
// and tcgen05.mma kind::f16 accumulates the whole K loop of a tile in TMEM, so
// the epilogue runs once per tile.  f16 keeps 11 significant bits (relative
// 2^-12 per operand; values here stay far inside its range); products
// accumulate in fp32.
//
// Same "swap AB" orientation as the e4m3 kernels: MMA M = 128 weight rows,
// N = BN tokens.  One pipeline stage is one 64-element K atom (128 bytes of
// f16 per row).  GEMM1 (KIND 1) holds the X1 and X2 rows of 128 features, so
// SwiGLU runs in the epilogue; GEMM2 (KIND 2) writes fp32 rows for the combine.
// Scheduling is the persistent stream-K of the e4m3 kernels; a split tile's
// partial sums are published to global memory and added, in fixed CTA order,
// by the last contributor.
//
// Warp roles: 0 TMA producer, 1 TMEM owner + MMA issuer, 2..2+NCONV-1 weight
// converters, the last four the epilogue.
#include "kernels.cuh"

namespace moe {


// Shared memory holds two rings:
//   raw ring (RS stages): what TMA writes -- the e4m3 weight tile(s) and the
//     f16 token tile; a stage is free once the MMA that read its tokens is done;
//   operand ring (OS stages): the converted f16 weight tile(s) the MMA reads.
// Only the raw ring waits on memory latency, so it gets most of the space:
// deeper prefetch for the same shared memory than one ring of whole stages.
// Weight conversion: e4m3 -> f16 by cvt (exact), then one f16 multiply by
// f16(s * 2^8), s the 128x128 block scale.  The 2^8 keeps small products out
// of the f16 subnormal range; the epilogue multiplies the fp32 accumulator by
// 2^-8 (exact).  Dequantised weights must stay below 2^8 in magnitude.  The
// scale's rounding to f16 adds at most 2^-11 relative to each weight block.
constexpr float kAccUnscale = 1.0f / 256.0f;

__device__ __forceinline__ void convert16(uint4 src, float scale, uint4& lo, uint4& hi) {
  const uint32_t w[4] = {src.x, src.y, src.z, src.w};
  const __half2 s2 = __float2half2_rn(scale * 256.0f);
  uint32_t out[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __nv_fp8x2_storage_t pair = static_cast<__nv_fp8x2_storage_t>((w[i] >> (16 * h)) & 0xFFFF);
      __half2 v = __hmul2(__half2(__nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3)), s2);
      out[i * 2 + h] = *reinterpret_cast<uint32_t*>(&v);
    }
  }
  lo = make_uint4(out[0], out[1], out[2], out[3]);
  hi = make_uint4(out[4], out[5], out[6], out[7]);
}

template <int KIND, int BN, int RS, int OS>
struct B16Cfg {
  static constexpr int NW = KIND == 1 ? 2 : 1;              // weight tiles (X1, X2) per stage
  static constexpr int K = KIND == 1 ? kHidden : kInter;    // reduction length
  static constexpr int ATOMS = K / 64;                      // pipeline iterations per tile
  static constexpr int NT = KIND == 1 ? kInter / 128 : kHidden / 128;
  static constexpr int W_ROWS = KIND == 1 ? kGemm1Out : kHidden;
  static constexpr int W8_TILE = 128 * 64;                  // e4m3 staging: 128 rows x 64 B
  static constexpr int W16_TILE = 128 * 128;                // f16: 128 rows x 128 B (swizzled)
  static constexpr int B_TILE = BN * 128;                   // f16 tokens: BN rows x 128 B
  static constexpr int OFF_B = NW * W8_TILE;               // token tile inside a raw stage
  static constexpr int RAW = OFF_B + B_TILE;                // raw stage bytes
  static constexpr int OPS = NW * W16_TILE;                 // operand stage bytes
  static constexpr int OFF_OP = RS * RAW;                   // operand ring after the raw ring
  static constexpr int ACC = NW * BN;                       // TMEM columns of one tile accumulator
  // Two accumulators (the epilogue of one tile overlaps the next tile's MMAs)
  // when they fit in TMEM's 512 columns, else one.
  static constexpr int NACC = 2 * ACC <= 512 ? 2 : 1;
  static constexpr int TMEM_COLS = NACC * ACC <= 128 ? 128 : NACC * ACC <= 256 ? 256 : 512;
  static constexpr int NCONV = 8;               // converter warps
  static constexpr int EPI0 = 64 + 32 * NCONV;              // first epilogue thread
  static constexpr int THREADS = EPI0 + 128;
  static constexpr int CROWS = 128 / NCONV;                 // weight rows per converter warp
  static_assert(CROWS % 8 == 0, "converter rows");
  static constexpr int SMEM = 1024 + RS * RAW + OS * OPS + 1024;
  static_assert(RAW % 1024 == 0 && OPS % 1024 == 0, "1024-byte aligned stages");
  static_assert(ACC <= 512, "TMEM accumulator");
  static_assert(BN % 16 == 0 && BN <= 256, "MMA N");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

// Instruction descriptor for kind::f16: A = B = f16, D = f32, K-major, M = 128.
__host__ __device__ constexpr uint32_t make_idesc_f16(int m, int n) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <int KIND, int BN, int RS, int OS>
__global__ void __launch_bounds__(B16Cfg<KIND, BN, RS, OS>::THREADS, 1)
moe_gemm_f16_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_b,
                     const GemmParams p) {
  using C = B16Cfg<KIND, BN, RS, OS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* aux = smem + C::OFF_OP + OS * C::OPS;
  uint64_t* full = reinterpret_cast<uint64_t*>(aux);       // TMA bytes of raw stage s landed
  uint64_t* empty = full + RS;                              // MMA finished with raw stage s
  uint64_t* conv = empty + RS;                              // converters wrote operand stage o
  uint64_t* opempty = conv + OS;                            // MMA finished with operand stage o
  uint64_t* accf = opempty + OS;                            // accumulator b complete
  uint64_t* acce = accf + 2;                                // accumulator b drained
  uint64_t* drain = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* last_flag = const_cast<int*>(abort_flag) + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  griddep_wait();
  griddep_launch_dependents();
  const WorkSched sch = make_work_sched(p.sched[KIND - 1], C::NT, C::ATOMS);
  const int n_iter = sch.n_iter();
  if (n_iter == 0) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < RS; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int o = 0; o < OS; ++o) { mbar_init(&conv[o], C::NCONV); mbar_init(&opempty[o], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&accf[b], 1); mbar_init(&acce[b], 4); }
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
    // ------------------------------------------------------------ TMA producer
    if (elect_one_lane()) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_b = l2_policy_evict_last();
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < n_iter; ++i) {
        int u, a, r;
        sch.at(i, C::ATOMS, u, a, r);
        const int2 mn = unit_tile(u, sch.n_mt, C::NT);
      const int mt = mn.x, nt = mn.y;
        const int4 tile = p.tiles[mt];
        const int s = i % RS;
        if (!mbar_wait_bounded(&empty[s], ((i / RS) & 1) ^ 1, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(&full[s], C::OFF_B + p.box_rows * 128);
        uint8_t* st = smem + s * C::RAW;
        // weights: e4m3 [rows][64 B] per tile (X1 then X2 for GEMM1)
        tma_load_3d(&tm_w, &full[s], st, 0, a, tile.x * C::W_ROWS + nt * 128, pol_w);
        if (KIND == 1)
          tma_load_3d(&tm_w, &full[s], st + C::W8_TILE, 0, a, tile.x * C::W_ROWS + kInter + nt * 128, pol_w);
        // tokens: f16 [BN rows][64 elements], 128-byte swizzle
        tma_load_3d(&tm_b, &full[s], st + C::OFF_B, 0, a, tile.y, pol_b);
        ++issued;
      }
      if (!ok) {
        raise_error(p.err, kDevTimeoutProducer);
        for (int i = max(0, issued - RS); i < issued; ++i) {
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[i % RS], (i / RS) & 1) &&
                 globaltimer_ns() - t0 < kWaitLimitNs / 10) {}
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one_lane()) {
      const uint32_t smem_base = smem_u32(smem);
      uint32_t idesc = 0;
      bool ok = true;
      int seg = 0;                      // segments (tile shares) started so far
      for (int i = 0; i < n_iter && ok; ++i) {
        int u, a, r;
        sch.at(i, C::ATOMS, u, a, r);
        const bool seg_first = (i == sch.n1) || (a == 0);
        const bool seg_last = (a == C::ATOMS - 1) || (i == n_iter - 1);
        const int b = seg % C::NACC;
        if (seg_first) {   // MMA N covers the tile's rows only
          const int rows = p.tiles[unit_tile(u, sch.n_mt, C::NT).x].z;
          idesc = make_idesc_f16(128, min(BN, (rows + 15) & ~15));
        }
        if (seg_first &&
            !mbar_wait_bounded(&acce[b], ((seg / C::NACC) & 1) ^ 1, abort_flag)) { ok = false; break; }
        // The converters waited for raw stage s before writing operand stage o,
        // so conv[o] also orders the token tile's TMA writes before the MMA.
        const int s = i % RS, o = i % OS;
        if (!mbar_wait_bounded(&conv[o], (i / OS) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint64_t bdesc = make_sdesc_sw128(smem_base + s * C::RAW + C::OFF_B);
        const uint32_t op = smem_base + C::OFF_OP + o * C::OPS;
#pragma unroll
        for (int w = 0; w < C::NW; ++w) {
          const uint64_t adesc = make_sdesc_sw128(op + w * C::W16_TILE);
          const uint32_t d = tmem_base + (uint32_t)(b * C::ACC + w * BN);
#pragma unroll
          for (int k = 0; k < 4; ++k)   // 4 x K=16 per 128-byte atom; +32 B = +2 in addr>>4
            tc_mma_f16(d, adesc + 2 * k, bdesc + 2 * k, idesc, (seg_first && k == 0) ? 0u : 1u);
        }
        tc_commit(&empty[s]);
        tc_commit(&opempty[o]);
        if (seg_last) { tc_commit(&accf[b]); ++seg; }
      }
      if (!ok) raise_error(p.err, kDevTimeoutMma);
      tc_commit(drain);
      const unsigned long long t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {}
    }
  } else if (warp < 2 + C::NCONV) {
    // ------------------------------------------------------------ weight converters
    // Warp q converts rows CROWS*q.. of each weight tile: 8 rows per step,
    // 4 lanes per row, 16 e4m3 (one 16-byte load) per lane -> 32 bytes of f16.
    const int q = warp - 2;
    for (int i = 0; i < n_iter; ++i) {
      int u, a, r;
      sch.at(i, C::ATOMS, u, a, r);
      const int2 mn = unit_tile(u, sch.n_mt, C::NT);
      const int mt = mn.x, nt = mn.y;
      const int e = p.tiles[mt].x;
      const int s = i % RS, o = i % OS;
      float wsc[C::NW];
#pragma unroll
      for (int w = 0; w < C::NW; ++w) {
        const int nb = KIND == 1 ? nt + w * (kInter / 128) : nt;
        wsc[w] = __ldg(p.w_scale + ((size_t)e * (C::W_ROWS / 128) + nb) * (C::K / 128) + a / 2);
      }
      if (!mbar_wait_bounded(&full[s], (i / RS) & 1, abort_flag)) break;
      if (!mbar_wait_bounded(&opempty[o], ((i / OS) & 1) ^ 1, abort_flag)) break;
      const uint8_t* st = smem + s * C::RAW;
      uint8_t* opst = smem + C::OFF_OP + o * C::OPS;
      const int part = lane & 3;
#pragma unroll
      for (int w = 0; w < C::NW; ++w) {
        uint4 src[C::CROWS / 8];
#pragma unroll
        for (int rr = 0; rr < C::CROWS / 8; ++rr) {
          const int row = q * C::CROWS + rr * 8 + (lane >> 2);
          src[rr] = *reinterpret_cast<const uint4*>(st + w * C::W8_TILE + row * 64 + part * 16);
        }
#pragma unroll
        for (int rr = 0; rr < C::CROWS / 8; ++rr) {
          const int row = q * C::CROWS + rr * 8 + (lane >> 2);
          uint4 lo, hi;
          convert16(src[rr], wsc[w], lo, hi);
          uint8_t* dst = opst + w * C::W16_TILE + row * 128;
          *reinterpret_cast<uint4*>(dst + (((2 * part) ^ (row & 7)) * 16)) = lo;
          *reinterpret_cast<uint4*>(dst + (((2 * part + 1) ^ (row & 7)) * 16)) = hi;
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[o]);
    }
    if (*abort_flag) raise_error(p.err, kDevTimeoutProducer);
  } else {
    // ------------------------------------------------------------ epilogue
    const int et = threadIdx.x - C::EPI0;       // 0..127
    const int qq = warp & 3;                    // TMEM lane quarter of this warp
    const int f = qq * 32 + lane;               // weight row inside the tile
    const uint32_t lane_addr = (uint32_t)(qq * 32) << 16;
    int seg = 0;
    int seg_a0 = 0;
    for (int i = 0; i < n_iter; ++i) {
      int u, a, r;
      sch.at(i, C::ATOMS, u, a, r);
      if (i == sch.n1 || a == 0) seg_a0 = a;
      const bool seg_last = (a == C::ATOMS - 1) || (i == n_iter - 1);
      if (!seg_last) continue;
      const int2 mn = unit_tile(u, sch.n_mt, C::NT);
      const int mt = mn.x, nt = mn.y;
      const int4 tile = p.tiles[mt];
      const int b = seg % C::NACC;
      const bool got = mbar_wait_warp(&accf[b], (seg / C::NACC) & 1, abort_flag);
      if (named_bar_or(1, 128, !got || *abort_flag != 0)) break;
      tc_fence_after();
      const uint32_t acc0 = tmem_base + lane_addr + (uint32_t)(b * C::ACC);
      const bool full_tile = (seg_a0 == 0 && a == C::ATOMS - 1);
      bool finish = true;
      int c_lo = 0, c_hi = -1;
      if (!full_tile) {
        // publish this CTA's share: [slot][w][token][128 rows] fp32
        const int slot = sch.slot(blockIdx.x, r, C::ATOMS);
        float* mine = p.partials + ((size_t)(blockIdx.x * 2 + slot) * C::NW) * BN * 128;
#pragma unroll 1
        for (int w = 0; w < C::NW; ++w)
#pragma unroll 1
          for (int c0 = 0; c0 < tile.z; c0 += 16) {
            float v[16];
            tmem_ld16(acc0 + w * BN + c0, v);
            tmem_ld_wait();
#pragma unroll
            for (int x = 0; x < 16; ++x) __stcg(mine + ((size_t)w * BN + c0 + x) * 128 + f, v[x]);
          }
        __threadfence();
        c_lo = sch.first_cta(r, C::ATOMS);
        c_hi = sch.last_cta(r, C::ATOMS);
        named_bar_sync(1, 128);
        if (et == 0) {
          const int old = atomicAdd(p.counters + u, 1);
          last_flag[0] = (old == c_hi - c_lo) ? 1 : 0;
        }
        named_bar_sync(1, 128);
        finish = last_flag[0] != 0;
        if (finish) __threadfence();
      }
      if (finish) {
        // Column chunks of 16 tokens: full sums (TMEM, or published partials in
        // fixed CTA order), then the epilogue of this GEMM.
#pragma unroll 1
        for (int c0 = 0; c0 < tile.z; c0 += 16) {
          float v[C::NW][16];
          if (full_tile) {
#pragma unroll
            for (int w = 0; w < C::NW; ++w) tmem_ld16(acc0 + w * BN + c0, v[w]);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int w = 0; w < C::NW; ++w)
#pragma unroll
              for (int x = 0; x < 16; ++x) v[w][x] = 0.f;
            for (int c = c_lo; c <= c_hi; ++c) {
              const int cslot = sch.slot(c, r, C::ATOMS);
              const float* src = p.partials + ((size_t)(c * 2 + cslot) * C::NW) * BN * 128;
#pragma unroll
              for (int w = 0; w < C::NW; ++w)
#pragma unroll
                for (int x = 0; x < 16; ++x) v[w][x] += __ldcg(src + ((size_t)w * BN + c0 + x) * 128 + f);
            }
          }
#pragma unroll
          for (int x = 0; x < 16; ++x) {
            const int j = c0 + x;
            if (j >= tile.z) break;
            const size_t row = (size_t)(tile.y + j);
            if (KIND == 1) {
              const float x1 = v[0][x] * kAccUnscale, x2 = v[C::NW - 1][x] * kAccUnscale;
              const float cv = x2 * __frcp_rn(1.0f + __expf(-x2)) * x1;
              p.inter16[row * kInter + nt * 128 + f] = __float2half_rn(cv);
            } else {
              p.down[row * kHidden + nt * 128 + f] = v[0][x] * kAccUnscale;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[b]);
      ++seg;
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
// Host-side dispatch
// --------------------------------------------------------------------------
template <int KIND, int BN> struct B16Pick;   // raw stages RS, operand stages OS
template <> struct B16Pick<1, 128> { static constexpr int RS = 5, OS = 2; };
template <> struct B16Pick<1, 256> { static constexpr int RS = 3, OS = 2; };
template <> struct B16Pick<2, 128> { static constexpr int RS = 6, OS = 3; };
template <> struct B16Pick<2, 256> { static constexpr int RS = 4, OS = 3; };

#define MOE_B16_CASES(X) X(1, 128) X(1, 256) X(2, 128) X(2, 256)

template <int KIND, int BN>
static cudaError_t launch_f16_one(const CUtensorMap* tm_w, const CUtensorMap* tm_b, const GemmParams& p,
                                  int grid, cudaStream_t st) {
  using P = B16Pick<KIND, BN>;
  using C = B16Cfg<KIND, BN, P::RS, P::OS>;
  auto kern = moe_gemm_f16_kernel<KIND, BN, P::RS, P::OS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(grid), dim3(C::THREADS), C::SMEM, st, *tm_w, *tm_b, p);
}

size_t gemm_f16_partials_bytes(int kind, int bn, int grid) {
#define X(KD, BB) \
  if (kind == KD && bn == BB) return (size_t)grid * 2 * B16Cfg<KD, BB, 1, 1>::NW * BB * 128 * sizeof(float);
  MOE_B16_CASES(X)
#undef X
  return 0;
}

cudaError_t launch_gemm_f16(int kind, int bn, const CUtensorMap* tm_w, const CUtensorMap* tm_b,
                             const GemmParams& p, int grid, cudaStream_t st) {
#define X(KD, BB) \
  if (kind == KD && bn == BB) return launch_f16_one<KD, BB>(tm_w, tm_b, p, grid, st);
  MOE_B16_CASES(X)
#undef X
  return cudaErrorInvalidValue;
}

}  // namespace moe

