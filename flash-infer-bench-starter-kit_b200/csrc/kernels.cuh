// Launcher declarations shared by the translation units of the MoE layer.
#pragma once

#include "common.cuh"

#include <atomic>

namespace moe {

// Widest GEMM1 token tile that gathers its rows with tile::gather4 (after the
// fused front kernel); wider tiles load the permuted activation.
constexpr int kGatherMaxBN = 32;

// Work description read by the grouped GEMMs (written by scan_kernel).  Its
// size matters: every field is a kernel parameter, and a larger block made
// the 64-token GEMM1 spill registers, so a field one GEMM never reads may
// share a slot with the other GEMM's (seg / row_token).
struct GemmParams {
  const int4* tiles;          // (local expert, first row, rows, 0) per token tile
  const int32_t* sched;       // sched[0] = #tiles for GEMM1, sched[1] = #tiles for GEMM2
  const float* w_scale;       // GEMM1: [E_l, 32, 56]; GEMM2: [E_l, 56, 16]
  const float* b_scale;       // GEMM1: act_scale [56, R_cap]; GEMM2: inter_scale [16, R_cap]
  int32_t* counters;          // stream-K arrival counters, one per output tile
  int* ready;                 // per local expert: GEMM1 units finished (GEMM1 adds, GEMM2 waits)
  union {
    const int32_t* seg;         // GEMM2: per-expert row offsets (rows of expert e)
    // GEMM1 after the fused front kernel: token rows are gathered straight
    // from hidden_states (tm_b is a 128-byte x 1-row map of it, tile::gather4)
    // by this permuted-row -> token map, so the activation is never
    // materialised (compiled into the GEMM1 variants with token tiles of at
    // most kGatherMaxBN rows; the host uses the fused front kernel only for
    // those).  Shares its slot with seg, which GEMM1 does not read.
    const int32_t* row_token;
  };
  int bn_prev;                // GEMM2: GEMM1's token-tile width
  // e4m3 GEMM1 after the fused front kernel: front_sync[0] = 1 once the tile
  // lists are written, front_sync[1] counts front CTAs whose gather is done.
  // GEMM1 starts streaming weights at the first and reads activations after
  // the second reaches front_ctas (no grid-dependency wait).  nullptr: off.
  int* front_sync;
  int front_ctas;
  int early_start;            // GEMM2: start before GEMM1 completes (small batches)
  float* partials;            // stream-K partial tiles, [grid][2][NW][BN][128]
  uint8_t* inter;             // GEMM1 output: e4m3 [2*R_cap, 2048] (row pairs, or hi/lo planes)
  float* inter_scale;         // GEMM1 output: [16, R_cap]
  float* down;                // GEMM2 output: fp32 [R_cap, 7168]
  int* err;
  int R_cap;
};

// Persistent schedule of a grouped GEMM: units (token tile x weight tile, see
// unit_tile) of ITERS pipeline iterations each, over gridDim.x CTAs.
//   phase 1: floor(units / G) full waves; in wave w CTA c runs unit w*G + c,
//            so the CTAs running at one time cover G consecutive units, which
//            share token tiles and weight tiles in L2;
//   phase 2: the R < G remaining units, as one contiguous stream-K range of
//            ceil(R*ITERS / G) iterations per CTA.  A unit split between CTAs
//            is finished by its last contributor (fixed-order reduction).
struct WorkSched {
  int n_mt, units, Wf, n1, it0, it1, L;
  int G, gid;                 // workers (CTAs, or CTA pairs) and this worker's index
  __host__ __device__ __forceinline__ int n_iter() const { return n1 + it1 - it0; }
  // Local iteration i -> unit u, iteration a inside the unit, and the unit's
  // phase-2 index r (-1 in phase 1: never split).
  __host__ __device__ __forceinline__ void at(int i, int ITERS, int& u, int& a, int& r) const {
    if (i < n1) {
      u = (i / ITERS) * G + gid;
      a = i % ITERS;
      r = -1;
    } else {
      const int it = it0 + i - n1;
      r = it / ITERS;
      a = it % ITERS;
      u = Wf * G + r;
    }
  }
  __host__ __device__ __forceinline__ int unit_of(int i, int ITERS) const {
    int u, a, r;
    at(i, ITERS, u, a, r);
    return u;
  }
  // First and last worker contributing to phase-2 unit r.
  __host__ __device__ __forceinline__ int first_cta(int r, int ITERS) const { return (r * ITERS) / L; }
  __host__ __device__ __forceinline__ int last_cta(int r, int ITERS) const { return ((r + 1) * ITERS - 1) / L; }
  // Partial-tile slot worker c uses for phase-2 unit r: 0 for the unit its
  // range starts in, 1 for the one it ends in.
  __host__ __device__ __forceinline__ int slot(int c, int r, int ITERS) const {
    return r == (c * L) / ITERS ? 0 : 1;
  }
};

__host__ __device__ __forceinline__ WorkSched make_work_sched_for(int n_mt, int NT, int ITERS, int G, int gid) {
  WorkSched s;
  s.G = G;
  s.gid = gid;
  s.n_mt = n_mt;
  s.units = n_mt * NT;
  s.Wf = s.units / G;
  s.n1 = s.Wf * ITERS;
  const int total2 = (s.units - s.Wf * G) * ITERS;
  s.L = (total2 + G - 1) / G > 1 ? (total2 + G - 1) / G : 1;
  s.it0 = gid * s.L < total2 ? gid * s.L : total2;
  s.it1 = s.it0 + s.L < total2 ? s.it0 + s.L : total2;
  return s;
}

__device__ __forceinline__ WorkSched make_work_sched(int n_mt, int NT, int ITERS) {
  return make_work_sched_for(n_mt, NT, ITERS, (int)gridDim.x, (int)blockIdx.x);
}

// Per-kernel launch set-up (the dynamic shared memory opt-in, checks of the
// compiled kernel) done once per device and CUDA context instead of on every
// launch: `seen` is the kernel's own table, indexed by device.
constexpr int kMaxCachedDevices = 64;
void* current_cu_context();   // the calling thread's CUcontext, nullptr if none
template <typename SetUp>
cudaError_t once_per_context(std::atomic<void*>* seen, SetUp set_up) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  void* ctx = current_cu_context();
  if (dev < 0 || dev >= kMaxCachedDevices || ctx == nullptr) return set_up();
  if (seen[dev].load(std::memory_order_acquire) == ctx) return cudaSuccess;
  e = set_up();
  if (e == cudaSuccess) seen[dev].store(ctx, std::memory_order_release);
  return e;
}

size_t gemm_partials_bytes(int kind, int bn, int grid);
int gemm_k_per_stage(int kind, int bn);
int gemm_ctas_per_sm(int kind, int bn);
cudaError_t launch_gemm(int kind, int bn, const CUtensorMap* tm_w, const CUtensorMap* tm_b,
                        const GemmParams& p, int grid, cudaStream_t st);

// e4m3 GEMMs with tokens on the MMA's M side, for large batches (gemm_tm.cu).
size_t gemm_tm_partials_bytes(int grid);
int gemm_tm_k_per_stage(int kind);
int gemm_tm_units_per_tile(int kind);
int gemm_tm_scale_box_cols();
cudaError_t launch_gemm_tm(int kind, const CUtensorMap* tm_w, const CUtensorMap* tm_b, const CUtensorMap* tm_bs,
                           const CUtensorMap* tm_ws, const GemmParams& p, int grid, cudaStream_t st);


cudaError_t launch_route(bool from_ids, const float* logits, const void* bias, int T,
                         float scaling, int local_offset, int E_l, int32_t* ids, float* w,
                         uint8_t* masks8, int NB8p, int* err, cudaStream_t st);
cudaError_t launch_scan(const uint8_t* masks8, int NB8p, int32_t* bases, int NB, int E_l, int32_t* seg,
                        int bn1, int bn2, int4* tiles1, int4* tiles2, int32_t* sched,
                        int32_t* counters1, int nt1, int32_t* counters2, int nt2, int* ready,
                        cudaStream_t st);
cudaError_t launch_scatter(const int32_t* ids, const uint8_t* masks8, int NB8p, const int32_t* bases, int T,
                           int E_l, int local_offset, int R_cap, const void* hidden,
                           const float* hs_scale, int32_t* inv_row, int32_t* row_token,
                           uint8_t* act, float* act_scale, cudaStream_t st);
// Routing + row assignment + activation gather in one launch, T <= kFrontMaxTokens.
cudaError_t launch_front(const float* logits, const void* bias, int T, float scaling, int local_offset,
                         int E_l, int R_cap, int bn1, int bn2, int nt1, int nt2, const void* hidden,
                         const float* hs_scale, int32_t* ids, float* w, uint8_t* masks8, int NB8p,
                         int32_t* seg, int4* tiles1, int4* tiles2, int32_t* sched,
                         int32_t* counters1, int32_t* counters2, int* ready, int32_t* inv_row,
                         int32_t* row_token, uint8_t* act, float* act_scale, int* err, int* front_sync,
                         cudaStream_t st);
cudaError_t launch_combine(const float* down, const int32_t* inv_row, const float* w, int T,
                           void* out, float* out_f32, const int* front_sync, int* err, cudaStream_t st);

// Defined in api.cu: one full layer call on a caller-provided workspace.
int run_layer_with_workspace(const moe_fp8_ds_args* a, void* ws, uint64_t ws_bytes, void* stream,
                             bool routed);

}  // namespace moe
