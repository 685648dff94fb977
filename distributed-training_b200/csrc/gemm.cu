// Persistent tcgen05 GEMM for sm_100a with fused epilogues.
//
//   C[M,N] (+)= op(A)[M,K] . op(B)[K,N]      bf16 operands, fp32 accumulation in TMEM
//
// Replaces the reference's NumPy matmuls of the Linear layers (dtrain/nn.py:63-65,
// dtrain/autograd.py:102-109): forward Y = X W + b, backward dX = dY W^T and
// dW = X^T dY.  Operand layouts are chosen per call with the descriptor "major"
// bits, so no transpose is ever materialised:
//   forward : A = X  (K-major),  B = W stored (in,out)  -> MN-major
//   dX      : A = dY (K-major),  B = W stored (in,out)  -> K-major (W^T)
//   dW      : A = X  stored (tokens,in) -> MN-major,  B = dY (tokens,out) -> MN-major
//
// Structure (one CTA per SM, persistent over output tiles, 10 warps):
//   warp 0      TMA producer: 128x64 A tile and BNx64 B tile per stage into
//               128B-swizzled shared memory, one mbarrier per stage.
//   warp 1      owns TMEM (2*BN columns = two accumulators); one lane issues
//               tcgen05.mma (M=128, N=BN, K=16) for every stage, then
//               tcgen05.commit to free the stage / publish the accumulator.
//   warps 2..9  epilogue, two warps per TMEM lane quarter, each owning half of
//               the tile's columns: tcgen05.ld 64 columns per wait, fused math
//               (bias, residual, GELU / GELU', scale), bf16/fp32 packing into a
//               per-warp shared-memory slab, then a TMA bulk-tensor store (or
//               TMA reduce-add for fp32 accumulation) that writes whole lines and
//               clips partial tiles in hardware.
// The two TMEM accumulators let the epilogue of tile i overlap the main loop of
// tile i+1.  Every barrier wait is bounded (common.cuh).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <mutex>

#include "common.cuh"

namespace dtb {

enum GemmEpi : int {
  EPI_BF16 = 0,     // out(bf16) = alpha*acc [+ bias] [+ resid]
  EPI_GELU = 1,     // aux(bf16) = acc + bias ; out(bf16) = gelu(aux)
  EPI_DGELU = 2,    // out(bf16) = acc * gelu'(aux)
  EPI_F32 = 3,      // out(f32)  = alpha*acc [+ out if accumulate]
  EPI_PARTIAL = 4,  // ws[split](f32) = acc   (split-K partial, reduced by splitk_reduce)
  EPI_LSE = 5,      // out(bf16) = acc, plus per (row, half-tile) softmax partials (max, sum exp) of the
                    // bf16-rounded outputs -> lse_part (the LM head fused with the cross-entropy forward)
};

// All-gather fused into the GEMM (ZeRO-1 forward): B is a weight stored in a flat bf16
// buffer partitioned over the ranks with the reference's partition rule
// (dtrain/comm.py:220-226); each rank's own partition is current and the rest is
// pulled from the owners' peer-mapped copies by the gather warps, k-block by k-block,
// while the MMA pipeline consumes the k-blocks already in place.
constexpr int kGatherRanks = 8;
constexpr int kGatherMaxKb = 128;   // K <= 8192
constexpr int kGatherWarps = 2;
// state[] layout (int32): [0, 128) per-k-block arrival counters, then
enum : int { GS_TICKET = 128, GS_DONE = 129, GS_FAIL = 130, GS_GEN = 131, GS_SITES = 256 };

struct GatherArgs {
  const bf16* peer[kGatherRanks];  // every rank's copy of B[0][0] (peer-mapped)
  bf16* local;                     // this rank's copy (the TMA source)
  long woff;                       // flat index of B[0][0] in the partitioned buffer
  long nflat;                      // elements of the partitioned buffer
  int rank, world;
  int sub;                         // work units per k-block
  int site;                        // this weight's slot in state[GS_SITES + site]
  int* state;
};

struct GemmArgs {
  GatherArgs g;
  int M, N, K;
  int epi;
  int splits;        // split-K factor (>= 1)
  const bf16* bias;  // [N] or nullptr
  const bf16* resid;
  long ldr;
  const bf16* aux_in;  // DGELU: pre-activation to differentiate
  long ldx;
  float alpha;
  int accumulate;
  float2* lse_part;  // EPI_LSE: [M, lse_np] (max, sum of exp(x - max)) per row and column half-tile
  int lse_np;
};

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + kEpiWarps * 32;
constexpr int kEpiSlab = 4096;  // bytes of store staging per epilogue warp (32 rows x 32 fp32)

template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : 5;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int EPI_BYTES = kEpiWarps * kEpiSlab;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ void tile_coords(int t, int mt, int nt, int& mi, int& ni) {
  // Group 16 M-tiles together so CTAs running concurrently share B (and A) tiles in L2.
  const int G = 16;
  const int per_group = G * nt;
  const int g = t / per_group;
  const int first = g * G;
  const int gm = min(G, mt - first);
  const int r = t - g * per_group;
  mi = first + r % gm;
  ni = r / gm;
}

__device__ __forceinline__ void load_bf16x8(const bf16* src, float* v) {
  uint4 u = *reinterpret_cast<const uint4*>(src);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// Load 32 bf16 values [col, col+32) of a row into fp32 (zeros past n_valid).
__device__ __forceinline__ void load_row32(const bf16* rowp, int col, int N, float* v) {
  if (col + 32 <= N) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) load_bf16x8(rowp + col + j, v + j);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (col + j < N) ? bf2f(rowp[col + j]) : 0.f;
  }
}

// Staging slabs hold one 32x32 output chunk, one row per lane, in the layout of the
// TMA store's swizzle mode, so that a warp's 16-byte stores hit distinct banks:
//   bf16 rows (64 B, SWIZZLE_64B):   16-byte unit j of row r sits at unit j ^ ((r >> 1) & 3)
//   fp32 rows (128 B, SWIZZLE_128B): 16-byte unit j of row r sits at unit j ^ (r & 7)
// (unswizzled rows 64 / 128 B apart put 8 lanes of a store phase on 2 / 1 bank groups:
// 4- and 8-way conflicts).  Slabs start on 2 KB boundaries, a multiple of both
// patterns' periods (512 B and 1 KB), as the swizzled TMA store requires.
__device__ __forceinline__ int slab_unit_bf16(int lane, int j) { return j ^ ((lane >> 1) & 3); }
__device__ __forceinline__ int slab_unit_f32(int lane, int j) { return j ^ (lane & 7); }

// Write 32 fp32 values as bf16 into this lane's 64-byte row of a slab.
__device__ __forceinline__ void slab_put_bf16(uint8_t* slab, int lane, const float* v) {
  uint4* dst = reinterpret_cast<uint4*>(slab + lane * 64);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 u;
    u.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
    u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
    u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
    u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
    dst[slab_unit_bf16(lane, j)] = u;
  }
}

__device__ __forceinline__ void slab_put_f32(uint8_t* slab, int lane, const float* v) {
  float4* dst = reinterpret_cast<float4*>(slab + lane * 128);
#pragma unroll
  for (int j = 0; j < 8; ++j)
    dst[slab_unit_f32(lane, j)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

// Epilogues whose chunk is one 32x32 bf16 tile (2 KB) stage alternate chunks in the
// two halves of the warp's 4 KB slab; fp32 and GELU (two outputs) chunks fill it.
__device__ __forceinline__ bool epi_double_buffered(int epi) {
  return epi == EPI_BF16 || epi == EPI_DGELU || epi == EPI_LSE;
}

__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// EPI_LSE (the head GEMM carrying the cross-entropy forward's row statistics,
// dtrain/autograd.py:250-266): fold 32 outputs of this lane's row (columns col..col+31, those < N) into
// the running (max m, sum s of exp(x - m)).  v holds the bf16-rounded outputs (epi_chunk
// rounds them), the values the logits tensor holds.  One exp2 per element plus two per chunk.
__device__ __forceinline__ void lse_fold(const float* v, int col, int N, float& m, float& s) {
  constexpr float kLog2e = 1.4426950408889634f;
  float x[32];
  float cm = -INFINITY;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    x[j] = (col + j < N) ? v[j] : -INFINITY;
    cm = fmaxf(cm, x[j]);
  }
  if (cm == -INFINITY) return;
  const float nb = -cm * kLog2e;
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    s0 += ex2_fast(fmaf(x[j], kLog2e, nb));
    s1 += ex2_fast(fmaf(x[j + 1], kLog2e, nb));
  }
  const float cs = s0 + s1;
  if (m == -INFINITY) { m = cm; s = cs; }
  else if (cm > m) { s = s * ex2_fast((m - cm) * kLog2e) + cs; m = cm; }
  else { s += cs * ex2_fast((cm - m) * kLog2e); }
}

// Before packing a chunk: lane 0 waits until the store that last used this (sub-)slab
// has read it - with two halves that is every store but the most recent one.
__device__ __forceinline__ void epi_slab_acquire(int lane, bool dbl) {
  if (lane == 0) {
    if (dbl) bulk_wait_read1();
    else bulk_wait_read0();
  }
  __syncwarp();
}

// Epilogue for one 32x32 chunk held in registers (this lane = one row).  Writes the
// staging slab and lets lane 0 issue the TMA store(s).
__device__ __forceinline__ void epi_chunk(const GemmArgs& a, const CUtensorMap* tmOut, const CUtensorMap* tmAux,
                                          uint8_t* slab, int lane, int row0, int col, int split, float* v) {
  const int row = row0 + lane;
  const bool row_ok = row < a.M;
  switch (a.epi) {
    case EPI_LSE: {
      // pack to bf16 once; v keeps the rounded values (unpacked with shifts, not
      // conversions) for the softmax statistics folded in by the caller
      uint4* dst = reinterpret_cast<uint4*>(slab + lane * 64);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t u[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          u[e] = pack_bf16x2(v[8 * j + 2 * e], v[8 * j + 2 * e + 1]);
          v[8 * j + 2 * e] = __uint_as_float(u[e] << 16);
          v[8 * j + 2 * e + 1] = __uint_as_float(u[e] & 0xffff0000u);
        }
        dst[slab_unit_bf16(lane, j)] = make_uint4(u[0], u[1], u[2], u[3]);
      }
      break;
    }
    case EPI_BF16: {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= a.alpha;
      if (a.bias) {
        float b[32];
        load_row32(a.bias, col, a.N, b);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += b[j];
      }
      if (a.resid && row_ok) {
        float r[32];
        load_row32(a.resid + (long)row * a.ldr, col, a.N, r);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += r[j];
      }
      slab_put_bf16(slab, lane, v);
      break;
    }
    case EPI_GELU: {
      if (a.bias) {
        float b[32];
        load_row32(a.bias, col, a.N, b);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += b[j];
      }
      // the saved pre-activation is the bf16-rounded value; GELU is taken of exactly that
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = bf2f(f2bf(v[j]));
      slab_put_bf16(slab, lane, v);  // aux chunk at slab[0, 2048)
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = gelu_fast(v[j]);
      slab_put_bf16(slab + 2048, lane, v);  // out chunk at slab[2048, 4096)
      break;
    }
    case EPI_DGELU: {
      if (row_ok) {
        float h[32];
        load_row32(a.aux_in + (long)row * a.ldx, col, a.N, h);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] *= gelu_grad_fast(h[j]);
      }
      slab_put_bf16(slab, lane, v);
      break;
    }
    case EPI_F32: {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= a.alpha;
      slab_put_f32(slab, lane, v);
      break;
    }
    case EPI_PARTIAL: {
      slab_put_f32(slab, lane, v);
      break;
    }
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (a.epi == EPI_GELU) {
      tma_store_2d(tmAux, slab, col, row0);
      tma_store_2d(tmOut, slab + 2048, col, row0);
    } else if (a.epi == EPI_PARTIAL) {
      tma_store_3d(tmOut, slab, col, row0, split);
    } else if (a.epi == EPI_F32 && a.accumulate) {
      tma_reduce_add_2d(tmOut, slab, col, row0);
    } else {
      tma_store_2d(tmOut, slab, col, row0);
    }
    bulk_commit();
  }
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void gather_bar() {
  asm volatile("bar.sync 1, %0;" ::"r"(kGatherWarps * 32) : "memory");
}

// [lo, hi) of partition c of n elements over W ranks (first n % W get one more).
__device__ __forceinline__ void part_bounds(long n, int W, int c, long& lo, long& hi) {
  const long base = n / W, extra = n % W;
  lo = c * base + min((long)c, extra);
  hi = lo + base + (c < extra ? 1 : 0);
}

// Copy B elements [s, e) (indices relative to B[0][0]) from src to dst with the
// gather warps: 16-byte peer loads, eight in flight per thread, scalar edges.
__device__ __forceinline__ void gather_copy(const bf16* __restrict__ src, bf16* __restrict__ dst, long s, long e,
                                            int t) {
  constexpr int NT = kGatherWarps * 32;
  const long vs = min(e, (s + 7) & ~7L), ve = max(vs, e & ~7L);
  for (long i = s + t; i < vs; i += NT) dst[i] = src[i];
  for (long i = ve + t; i < e; i += NT) dst[i] = src[i];
  const uint4* s4 = reinterpret_cast<const uint4*>(src + vs);
  uint4* d4 = reinterpret_cast<uint4*>(dst + vs);
  const long nv = (ve - vs) >> 3;
  constexpr int U = 8;  // 8 KB in flight per CTA covers the NVLink load latency at ~770 GB/s over 148 SMs
  long i = t;
  for (; i + (U - 1) * NT < nv; i += U * NT) {
    uint4 r[U];
#pragma unroll
    for (int j = 0; j < U; ++j) r[j] = __ldcg(s4 + i + j * NT);
#pragma unroll
    for (int j = 0; j < U; ++j) d4[i + j * NT] = r[j];
  }
  for (; i < nv; i += NT) d4[i] = __ldcg(s4 + i);
}

// ---- in-GEMM all-gather roles, shared by the 1-SM and 2-SM kernels ----------
// Thread 0 at set-up: the generation to pull (0: the weight is already current).
// Only the grid's last CTA updates the site's generation (at exit), so every CTA
// reads the same pair here.
__device__ __forceinline__ int gather_generation(const GatherArgs& g) {
  const int need = *reinterpret_cast<volatile int*>(g.state + GS_GEN);
  const int have = *reinterpret_cast<volatile int*>(g.state + GS_SITES + g.site);
  return (need != have) ? need : 0;
}

// TMA producer: before the first B load of k-block kb, wait (bounded) until every
// work unit of that k-block has landed in local memory.  `ready_lo/hi` remember the
// k-blocks already seen complete.  Returns false on timeout or abort.
__device__ __forceinline__ bool gather_wait_kb(const GatherArgs& g, int kb, uint64_t& ready_lo, uint64_t& ready_hi,
                                               volatile int* abort_flag) {
  if ((((kb < 64) ? ready_lo : ready_hi) >> (kb & 63)) & 1ull) return true;
  const int* cnt = g.state + kb;
  if (ld_acquire_gpu(cnt) < g.sub) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
      if (ld_acquire_gpu(cnt) >= g.sub) break;
      if ((i & 63u) == 0u) {
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > kPipeWaitNs) {
          set_status(kStatusMbarTimeout);
          *abort_flag = 1;
          return false;
        }
      }
    }
  }
  // generic-proxy stores of other CTAs -> this CTA's TMA (async proxy) reads
  fence_proxy_async_global();
  if (kb < 64) ready_lo |= 1ull << kb;
  else ready_hi |= 1ull << (kb & 63);
  return true;
}

// Gather warps: work units (k-block kb, piece) are handed out by a grid-wide ticket
// in k-block order, so whichever CTAs are resident pull the earliest k-blocks first
// and no CTA waits on a CTA that has not started.
__device__ __forceinline__ void gather_worker(const GatherArgs& g, int K, int N, int kb_total, int gt) {
  __shared__ int s_ticket;
  const int total = kb_total * g.sub;
  for (;;) {
    if (gt == 0) s_ticket = atomicAdd(g.state + GS_TICKET, 1);
    gather_bar();
    const int u = s_ticket;
    gather_bar();
    if (u >= total) break;
    const int kb = u / g.sub, pc = u - kb * g.sub;
    const long r1 = min((long)K, (long)(kb + 1) * kBK);
    const long e0 = (long)kb * kBK * N, e1 = r1 * N;
    const long step = ((((e1 - e0) + g.sub - 1) / g.sub) + 7) & ~7L;
    const long s = min(e1, e0 + pc * step), e = min(e1, s + step);
    for (int p = 0; p < g.world; ++p) {
      if (p == g.rank) continue;
      long lo, hi;
      part_bounds(g.nflat, g.world, p, lo, hi);
      const long a0 = max(s, lo - g.woff), a1 = min(e, hi - g.woff);
      if (a0 < a1) gather_copy(g.peer[p], g.local, a0, a1, gt);
    }
    fence_proxy_async_global();
    gather_bar();
    if (gt == 0) {
      __threadfence();
      atomicAdd(g.state + kb, 1);
    }
  }
}

// Thread 0 at exit: the last CTA to leave resets the counters for the next launch
// and records that this call site now holds generation `gen` (unless a wait failed).
__device__ __forceinline__ void gather_exit(const GatherArgs& g, int kb_total, int gen, bool aborted) {
  int* st = g.state;
  if (aborted) atomicOr(st + GS_FAIL, 1);
  __threadfence();
  if (atomicAdd(st + GS_DONE, 1) == (int)gridDim.x - 1) {
    __threadfence();
    volatile int* vs = st;
    for (int i = 0; i < kb_total; ++i) vs[i] = 0;
    vs[GS_TICKET] = 0;
    if (gen != 0 && vs[GS_FAIL] == 0) vs[GS_SITES + g.site] = gen;
    vs[GS_FAIL] = 0;
    vs[GS_DONE] = 0;
    __threadfence();
  }
}

template <int BN, bool A_MN, bool B_MN, bool GATHER = false>
__global__ void __maxnreg__(DTB_CORESIDENT_MAXNREG)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmAux,
                   GemmArgs args) {
  using Cfg = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_smem = smem + Cfg::STAGES * Cfg::STAGE_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(epi_smem + Cfg::EPI_BYTES);
  uint64_t* empty_bar = full_bar + Cfg::STAGES;
  uint64_t* tfull_bar = empty_bar + Cfg::STAGES;  // [2]
  uint64_t* tempty_bar = tfull_bar + 2;           // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* gather_gen = abort_flag + 1;  // GATHER: generation to reach, 0 = nothing to pull

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], kEpiWarps);
    }
    *abort_flag = 0;
    if (GATHER) *gather_gen = gather_generation(args.g);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int M = args.M, N = args.N, K = args.K;
  const int mt = (M + kBM - 1) / kBM;
  const int nt = (N + BN - 1) / BN;
  const int kb_total = (K + kBK - 1) / kBK;
  const int splits = args.splits;
  const int units = mt * nt * splits;
  const bool gathering = GATHER && *gather_gen != 0;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint64_t ready_lo = 0, ready_hi = 0;  // GATHER: k-blocks known to be in place (kb < 128)
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int t = u / splits, sp = u % splits;
        int mi, ni;
        tile_coords(t, mt, nt, mi, ni);
        const int m0 = mi * kBM, n0 = ni * BN;
        const int kb0 = (int)((long)kb_total * sp / splits), kb1 = (int)((long)kb_total * (sp + 1) / splits);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (GATHER && gathering && !gather_wait_kb(args.g, kb, ready_lo, ready_hi, abort_flag)) {
            ok = false;
            break;
          }
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag)) { ok = false; break; }
          uint8_t* sA = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sB = sA + Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
          const int k0 = kb * kBK;
          if (!A_MN) {
            tma_load_2d(&tmA, sA, &full_bar[stage], k0, m0);
          } else {
#pragma unroll
            for (int c = 0; c < kBM / 64; ++c) tma_load_2d(&tmA, sA + c * 8192, &full_bar[stage], m0 + c * 64, k0);
          }
          if (!B_MN) {
            tma_load_2d(&tmB, sB, &full_bar[stage], k0, n0);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_2d(&tmB, sB + c * 8192, &full_bar[stage], n0 + c * 64, k0);
          }
          if (++stage == Cfg::STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = make_idesc_bf16(kBM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int ab = 0;
      uint32_t aphase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int sp = u % splits;
        const int kb0 = (int)((long)kb_total * sp / splits), kb1 = (int)((long)kb_total * (sp + 1) / splits);
        if (!mbar_wait(&tempty_bar[ab], aphase ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(ab * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t aBase = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t bBase = aBase + Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // K-major: step 16 elements (32 B) inside the 128 B swizzle row.
            // MN-major: step 16 rows (2 KB) of the K dimension.
            const uint64_t ad = A_MN ? make_sw128_desc(aBase + kk * 2048, 8192, 1024)
                                     : make_sw128_desc(aBase + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_sw128_desc(bBase + kk * 2048, 8192, 1024)
                                     : make_sw128_desc(bBase + kk * 32, 16, 1024);
            tc_mma_f16(d_tmem, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&empty_bar[stage]);
          if (++stage == Cfg::STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(&tfull_bar[ab]);
        if (++ab == 2) { ab = 0; aphase ^= 1; }
      }
    }
  } else if (GATHER && warp >= 2 + kEpiWarps) {
    // -------------------------------------------------------------- gather warps
    if (gathering) gather_worker(args.g, K, N, kb_total, threadIdx.x - (2 + kEpiWarps) * 32);
  } else {
    // -------------------------------------------------------------- epilogue
    const int ew = warp - 2;       // 0..7
    const int q = warp & 3;        // TMEM lane quarter this warp may access
    const int half = ew >> 2;      // which half of the tile's columns
    uint8_t* slab = epi_smem + ew * kEpiSlab;
    // bf16 chunks (2 KB) alternate between the two halves of the slab, so the next
    // chunk is packed while the previous one's TMA store is still reading
    const bool dbl = epi_double_buffered(args.epi);
    constexpr int kSub = 2048;
    uint32_t ck = 0;
    int ab = 0;
    uint32_t aphase = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const int t = u / splits, sp = u % splits;
      int mi, ni;
      tile_coords(t, mt, nt, mi, ni);
      const int m0 = mi * kBM, n0 = ni * BN;
      if (!mbar_wait(&tfull_bar[ab], aphase, abort_flag)) break;
      tc_fence_after();
      const int row0 = m0 + q * 32;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BN);
      const int c_begin = half * (BN / 2), c_end = c_begin + BN / 2;
      float lm = -INFINITY, ls = 0.f;  // EPI_LSE running softmax statistics of this lane's row
#pragma unroll 1
      for (int c = c_begin; c < c_end; c += 64) {
        if (n0 + c >= N) break;  // warp-uniform
        uint32_t r0[32], r1[32];
        tmem_ld32_issue(tbase + c, r0);
        tmem_ld32_issue(tbase + c + 32, r1);
        tmem_wait_ld();
        float v[32];
        // chunk c .. c+31
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r0[j]);
        epi_slab_acquire(lane, dbl);  // the sub-slab's previous store has read its source
        epi_chunk(args, &tmOut, &tmAux, slab + (dbl ? (ck & 1) * kSub : 0), lane, row0, n0 + c, sp, v);
        if (args.epi == EPI_LSE) lse_fold(v, n0 + c, N, lm, ls);
        ++ck;
        // chunk c+32 .. c+63
        if (n0 + c + 32 < N) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r1[j]);
          epi_slab_acquire(lane, dbl);
          epi_chunk(args, &tmOut, &tmAux, slab + (dbl ? (ck & 1) * kSub : 0), lane, row0, n0 + c + 32, sp, v);
          if (args.epi == EPI_LSE) lse_fold(v, n0 + c + 32, N, lm, ls);
          ++ck;
        }
      }
      if (args.epi == EPI_LSE && row0 + lane < M) args.lse_part[(long)(row0 + lane) * args.lse_np + ni * 2 + half] =
          make_float2(lm, ls);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[ab]);
      if (++ab == 2) { ab = 0; aphase ^= 1; }
    }
    if (lane == 0) bulk_wait0();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
  if (GATHER && threadIdx.x == 0) gather_exit(args.g, kb_total, *gather_gen, *abort_flag != 0);
}

// -------------------------------------------------------------------------
// 2-SM variant: a cluster of two CTAs computes 256x256 output tiles with
// tcgen05 cta_group::2 (M=256, N=256, K=16 per instruction).  CTA r of the pair
// loads A rows [m0 + 128r, +128) and B columns [n0 + 128r, +128) into its own
// shared memory (32 KB per k-block instead of the 48 KB a 1-SM 128x256 tile
// needs), the leader's single MMA thread multiplies the pair's operands, and
// each CTA's TMEM receives its 128 rows of the 256x256 accumulator.  This halves
// B's shared-memory and L2 traffic per SM, which bounds the 1-SM mainloop.
// Barriers: full (leader; TMA bytes of both CTAs), empty / tile-full (both CTAs,
// arrived by the leader's multicast commit), tile-empty (leader; 2x8 epilogue
// warps, the peer's arrive remotely), done (end-of-kernel handshake).  Every
// wait is bounded; the only cluster barrier is the one after set-up.
struct Gemm2Cfg {
  static constexpr int A_BYTES = kBM * kBK * 2;        // 16 KB: this CTA's 128 rows
  static constexpr int B_BYTES = 128 * kBK * 2;        // 16 KB: this CTA's 128 columns
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 5;
  static constexpr int TMEM_COLS = 512;                // two 256-column accumulators
  static constexpr int EPI_BYTES = kEpiWarps * 2 * kEpiSlab;  // two 4 KB slabs per epilogue warp
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 + 256;
};

template <bool A_MN, bool B_MN, bool GATHER = false>
__global__ void __maxnreg__(DTB_CORESIDENT_MAXNREG)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmAux,
                    GemmArgs args) {
  using Cfg = Gemm2Cfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_smem = smem + Cfg::STAGES * Cfg::STAGE_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(epi_smem + Cfg::EPI_BYTES);
  uint64_t* empty_bar = full_bar + Cfg::STAGES;
  uint64_t* tfull_bar = empty_bar + Cfg::STAGES;  // [2]
  uint64_t* tempty_bar = tfull_bar + 2;           // [2]
  uint64_t* done_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* gather_gen = abort_flag + 1;  // GATHER: generation to reach, 0 = nothing to pull

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 2 * kEpiWarps);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    if (GATHER) *gather_gen = gather_generation(args.g);
    fence_barrier_init_cluster();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int M = args.M, N = args.N, K = args.K;
  const int mt = (M + 255) / 256;
  const int nt = (N + 255) / 256;
  const int kb_total = (K + kBK - 1) / kBK;
  const int splits = args.splits;
  const int units = mt * nt * splits;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const bool gathering = GATHER && *gather_gen != 0;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer (both CTAs)
      const uint32_t lead_full0 = mapa_shared(&full_bar[0], 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint64_t ready_lo = 0, ready_hi = 0;  // GATHER: k-blocks known to be in place
      for (int u = pair; u < units && ok; u += npairs) {
        const int t = u / splits, sp = u % splits;
        int mi, ni;
        tile_coords(t, mt, nt, mi, ni);
        const int m0 = mi * 256 + (int)rank * 128, n0 = ni * 256 + (int)rank * 128;
        const int kb0 = (int)((long)kb_total * sp / splits), kb1 = (int)((long)kb_total * (sp + 1) / splits);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (GATHER && gathering && !gather_wait_kb(args.g, kb, ready_lo, ready_hi, abort_flag)) {
            ok = false;
            break;
          }
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag)) { ok = false; break; }
          uint8_t* sA = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sB = sA + Cfg::A_BYTES;
          const uint32_t fb = lead_full0 + (uint32_t)(stage * sizeof(uint64_t));
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::STAGE_BYTES);
          const int k0 = kb * kBK;
          if (!A_MN) {
            tma_load_2d_pair(&tmA, sA, fb, k0, m0);
          } else {
            tma_load_2d_pair(&tmA, sA, fb, m0, k0);
            tma_load_2d_pair(&tmA, sA + 8192, fb, m0 + 64, k0);
          }
          if (!B_MN) {
            tma_load_2d_pair(&tmB, sB, fb, k0, n0);
          } else {
            tma_load_2d_pair(&tmB, sB, fb, n0, k0);
            tma_load_2d_pair(&tmB, sB + 8192, fb, n0 + 64, k0);
          }
          if (++stage == Cfg::STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer (leader only)
      constexpr uint32_t idesc = make_idesc_bf16(256, 256, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int ab = 0;
      uint32_t aphase = 0;
      bool ok = true;
      for (int u = pair; u < units && ok; u += npairs) {
        const int sp = u % splits;
        const int kb0 = (int)((long)kb_total * sp / splits), kb1 = (int)((long)kb_total * (sp + 1) / splits);
        if (!mbar_wait(&tempty_bar[ab], aphase ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(ab * 256);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t aBase = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t bBase = aBase + Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = A_MN ? make_sw128_desc(aBase + kk * 2048, 8192, 1024)
                                     : make_sw128_desc(aBase + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_sw128_desc(bBase + kk * 2048, 8192, 1024)
                                     : make_sw128_desc(bBase + kk * 32, 16, 1024);
            tc_mma_f16_pair(d_tmem, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          tc_commit_pair(&empty_bar[stage], 0x3);
          if (++stage == Cfg::STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit_pair(&tfull_bar[ab], 0x3);
        if (++ab == 2) { ab = 0; aphase ^= 1; }
      }
    }
  } else if (GATHER && warp >= 2 + kEpiWarps) {
    // -------------------------------------------------------------- gather warps (both CTAs)
    if (gathering) gather_worker(args.g, K, N, kb_total, threadIdx.x - (2 + kEpiWarps) * 32);
  } else {
    // -------------------------------------------------------------- epilogue (both CTAs)
    const int ew = warp - 2;
    const int q = warp & 3;
    const int half = ew >> 2;
    // two full slabs per warp: every epilogue (fp32, GELU's two outputs) packs chunk
    // i+1 while chunk i's TMA store is still reading
    uint8_t* slab = epi_smem + ew * 2 * kEpiSlab;
    const uint32_t lead_tempty0 = mapa_shared(&tempty_bar[0], 0);
    const bool dbl = true;
    constexpr int kSub = kEpiSlab;
    uint32_t ck = 0;
    int ab = 0;
    uint32_t aphase = 0;
    for (int u = pair; u < units; u += npairs) {
      const int t = u / splits, sp = u % splits;
      int mi, ni;
      tile_coords(t, mt, nt, mi, ni);
      const int m0 = mi * 256 + (int)rank * 128, n0 = ni * 256;
      if (!mbar_wait(&tfull_bar[ab], aphase, abort_flag)) break;
      tc_fence_after();
      const int row0 = m0 + q * 32;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * 256);
      const int c_begin = half * 128, c_end = c_begin + 128;
      float lm = -INFINITY, ls = 0.f;  // EPI_LSE running softmax statistics of this lane's row
#pragma unroll 1
      for (int c = c_begin; c < c_end; c += 64) {
        if (n0 + c >= N) break;  // warp-uniform
        uint32_t r0[32], r1[32];
        tmem_ld32_issue(tbase + c, r0);
        tmem_ld32_issue(tbase + c + 32, r1);
        tmem_wait_ld();
        float v[32];
        // chunk c .. c+31
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r0[j]);
        epi_slab_acquire(lane, dbl);  // the sub-slab's previous store has read its source
        epi_chunk(args, &tmOut, &tmAux, slab + (dbl ? (ck & 1) * kSub : 0), lane, row0, n0 + c, sp, v);
        if (args.epi == EPI_LSE) lse_fold(v, n0 + c, N, lm, ls);
        ++ck;
        // chunk c+32 .. c+63
        if (n0 + c + 32 < N) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r1[j]);
          epi_slab_acquire(lane, dbl);
          epi_chunk(args, &tmOut, &tmAux, slab + (dbl ? (ck & 1) * kSub : 0), lane, row0, n0 + c + 32, sp, v);
          if (args.epi == EPI_LSE) lse_fold(v, n0 + c + 32, N, lm, ls);
          ++ck;
        }
      }
      if (args.epi == EPI_LSE && row0 + lane < M) args.lse_part[(long)(row0 + lane) * args.lse_np + ni * 2 + half] =
          make_float2(lm, ls);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(lead_tempty0 + (uint32_t)(ab * sizeof(uint64_t)));
      if (++ab == 2) { ab = 0; aphase ^= 1; }
    }
    if (lane == 0) bulk_wait0();
    __syncwarp();
  }

  // Neither CTA releases the pair's TMEM before the other has finished with it.
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_cluster(mapa_shared(done_bar, rank ^ 1));
    mbar_wait(done_bar, 0, abort_flag);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
  if (GATHER && threadIdx.x == 0) gather_exit(args.g, kb_total, *gather_gen, *abort_flag != 0);
}

// Deterministic split-K reduction: out = alpha * sum_{s=0..S-1} ws[s] (+ out).
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int S, long MN, int N, float* out_f32,
                                     bf16* out_bf16, long ldo, float alpha, int accumulate) {
  long i = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i >= MN) return;
  float4 acc = *reinterpret_cast<const float4*>(ws + i);
  for (int s = 1; s < S; ++s) {
    float4 p = *reinterpret_cast<const float4*>(ws + (long)s * MN + i);
    acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
  }
  const long r = i / N, c = i % N;  // N % 4 == 0 is required by the host
  if (out_f32) {
    float4* o = reinterpret_cast<float4*>(out_f32 + r * ldo + c);
    float4 x = make_float4(acc.x * alpha, acc.y * alpha, acc.z * alpha, acc.w * alpha);
    if (accumulate) {
      float4 p = *o;
      x.x += p.x; x.y += p.y; x.z += p.z; x.w += p.w;
    }
    *o = x;
  } else {
    bf16* o = out_bf16 + r * ldo + c;
    o[0] = f2bf(acc.x * alpha); o[1] = f2bf(acc.y * alpha); o[2] = f2bf(acc.z * alpha); o[3] = f2bf(acc.w * alpha);
  }
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D bf16 operand map over a row-major matrix [rows, cols] with row stride ld (elements), 128B swizzle.
static CUtensorMap make_map(const void* base, long rows, long cols, long ld, int box_cols, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r);
  return m;
}

// Store map: [rows, cols] (optionally [depth, rows, cols]) row-major, 32x32 boxes, with
// the staging slabs' swizzle (64B for bf16 rows, 128B for fp32 rows).
static CUtensorMap make_store_map(void* base, bool f32, long rows, long cols, long ld, long depth = 0) {
  CUtensorMap m;
  const int esz = f32 ? 4 : 2;
  const CUtensorMapDataType dt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUtensorMapSwizzle sw = f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r;
  if (depth > 0) {
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)depth};
    cuuint64_t strides[2] = {(cuuint64_t)ld * esz, (cuuint64_t)ld * rows * esz};
    cuuint32_t box[3] = {32, 32, 1};
    r = get_encode_fn()(&m, dt, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        sw, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * esz};
    cuuint32_t box[2] = {32, 32};
    r = get_encode_fn()(&m, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        sw, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (store) failed with code ", (int)r);
  return m;
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, bool A_MN, bool B_MN, bool GATHER = false>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const CUtensorMap& tx,
                        const GemmArgs& a, cudaStream_t st) {
  using Cfg = GemmCfg<BN>;
  static bool attr_set = false;
  auto kern = gemm_tc_kernel<BN, A_MN, B_MN, GATHER>;
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
    attr_set = true;
  }
  const int mt = (a.M + kBM - 1) / kBM, nt = (a.N + BN - 1) / BN;
  const int units = mt * nt * a.splits;
  const int grid = std::min(units, num_sms());
  kern<<<grid, GATHER ? kThreads + kGatherWarps * 32 : kThreads, Cfg::SMEM_BYTES, st>>>(ta, tb, to, tx, a);
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static int max_pair_clusters() {
  static int n = -1;
  if (n < 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 74, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = Gemm2Cfg::SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaFuncSetAttribute(gemm_tc2_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         Gemm2Cfg::SMEM_BYTES);
    int c = 0;
    if (cudaOccupancyMaxActiveClusters(&c, gemm_tc2_kernel<false, true>, &cfg) != cudaSuccess || c <= 0) {
      cudaGetLastError();
      c = num_sms() / 2;
    }
    n = c;
  }
  return n;
}

template <bool A_MN, bool B_MN, bool GATHER = false>
static void launch_gemm2(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const CUtensorMap& tx,
                         const GemmArgs& a, cudaStream_t st) {
  static bool attr_set = false;
  auto kern = gemm_tc2_kernel<A_MN, B_MN, GATHER>;
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Gemm2Cfg::SMEM_BYTES);
    attr_set = true;
  }
  const int units = ((a.M + 255) / 256) * ((a.N + 255) / 256) * a.splits;
  const int pairs = std::min(units, max_pair_clusters());
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(GATHER ? kThreads + kGatherWarps * 32 : kThreads, 1, 1);
  cfg.dynamicSmemBytes = Gemm2Cfg::SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, to, tx, a));
  count_launch();
}

// Split-K factor for the 2-SM path: the same makespan model over pair tiles
// (256x256) and co-resident CTA pairs.
static int choose_splits2(int M, int N, int K, bool allow_split) {
  const int pairs = max_pair_clusters();
  const long tiles = (long)((M + 255) / 256) * ((N + 255) / 256);
  const int kb = (K + kBK - 1) / kBK;
  const double kb_seconds = 2.0 * 256 * 256 * kBK / (2 * 1.4e15 / num_sms());
  int splits = 1;
  double best = 1e30;
  for (int s = 1; s <= 16; ++s) {
    if (s > 1 && (!allow_split || kb / s < 8)) break;
    const long waves = (tiles * s + pairs - 1) / pairs;
    const double t = waves * (double)((kb + s - 1) / s) * kb_seconds +
                     (s > 1 ? (double)M * N * 4.0 * (s + 1) / 6.0e12 + 4e-6 : 0.0);
    if (t < best * 0.97) {
      best = t;
      splits = s;
    }
  }
  return splits;
}

// Picks the tile width and split-K factor.  128x256 tiles sustain ~1.4 PFLOP/s
// on the main loop while 128x128 tiles measured ~0.8, so BN=256 is used whenever
// N > 128.  The split-K factor s minimises a makespan model of the persistent
// grid: ceil(tiles*s / SMs) waves of ceil(kb/s) k-blocks each, plus the fp32
// partial traffic of the deterministic reduction ((s+1) M N 4 bytes) when s > 1.
static void choose_tiling(int M, int N, int K, int& bn, int& splits, bool allow_split = true) {
  const int sms = num_sms();
  const int mt = (M + kBM - 1) / kBM;
  bn = (N <= 128) ? 128 : 256;
  const int tiles = mt * ((N + bn - 1) / bn);
  const int kb = (K + kBK - 1) / kBK;
  const double kb_seconds = 2.0 * kBM * bn * kBK / (1.4e15 / sms);  // one k-block on one SM
  splits = 1;
  double best = 1e30;
  for (int s = 1; s <= 16; ++s) {
    if (s > 1 && (!allow_split || kb / s < 8)) break;
    const long waves = ((long)tiles * s + sms - 1) / sms;
    const double t = waves * (double)((kb + s - 1) / s) * kb_seconds +
                     (s > 1 ? (double)M * N * 4.0 * (s + 1) / 6.0e12 + 4e-6 : 0.0);
    if (t < best * 0.97) {
      best = t;
      splits = s;
    }
  }
}

// a: stored [M,K] (a_trans=false) or [K,M] (a_trans=true); b: stored [K,N] (b_trans=false) or [N,K] (b_trans=true).
// `gather` (forward GEMMs of ZeRO-1 only): B's peer partitions are pulled in the kernel.
// `lse_part` (EPI_LSE only): receives the [M, np, 2] softmax partials.
static void gemm_impl(torch::Tensor a, bool a_trans, torch::Tensor b, bool b_trans, torch::Tensor out, int64_t epi,
                      c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> resid,
                      c10::optional<torch::Tensor> aux, double alpha, bool accumulate, int64_t force_bn,
                      int64_t force_splits, c10::optional<torch::Tensor> workspace, const GatherArgs* gather,
                      torch::Tensor* lse_part = nullptr) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda(), "gemm: CUDA tensors expected");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm: bf16 operands expected");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "gemm: 2-D tensors expected");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && out.stride(1) == 1, "gemm: rows must be contiguous");
  const long M = a_trans ? a.size(1) : a.size(0);
  const long K = a_trans ? a.size(0) : a.size(1);
  const long Kb = b_trans ? b.size(1) : b.size(0);
  const long N = b_trans ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm: inner dimensions differ (", K, " vs ", Kb, ")");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm: output shape mismatch");
  TORCH_CHECK(M > 0 && N > 0 && K > 0, "gemm: empty problem");
  TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0, "gemm: leading dimensions must be multiples of 8");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(a.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(b.data_ptr()) & 15) == 0,
              "gemm: operands must be 16-byte aligned");
  TORCH_CHECK(N % 8 == 0 && out.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0,
              "gemm: output columns / leading dimension must be multiples of 8 and 16-byte aligned");
  const bool f32_out = (epi == EPI_F32);
  TORCH_CHECK(out.scalar_type() == (f32_out ? at::kFloat : at::kBFloat16), "gemm: wrong output dtype for epilogue");
  TORCH_CHECK((epi >= EPI_BF16 && epi <= EPI_F32) || (epi == EPI_LSE && lse_part), "gemm: unknown epilogue");
  TORCH_CHECK(epi != EPI_LSE || (!a_trans && !(bias && bias->defined()) && !(resid && resid->defined()) &&
                                 !accumulate && alpha == 1.0),
              "gemm: the softmax-statistics epilogue is a plain forward X @ W");
  c10::cuda::CUDAGuard guard(a.device());
  bind_device_context(a.get_device());

  GemmArgs args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.epi = (int)epi;
  args.alpha = (float)alpha;
  args.accumulate = accumulate ? 1 : 0;
  if (bias && bias->defined()) {
    TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == N && bias->is_contiguous(), "gemm: bias");
    args.bias = reinterpret_cast<const bf16*>(bias->data_ptr());
  }
  if (resid && resid->defined()) {
    TORCH_CHECK(resid->scalar_type() == at::kBFloat16 && resid->size(0) == M && resid->size(1) == N &&
                    resid->stride(1) == 1 && resid->stride(0) % 8 == 0,
                "gemm: resid");
    args.resid = reinterpret_cast<const bf16*>(resid->data_ptr());
    args.ldr = resid->stride(0);
  }
  torch::Tensor auxt;
  if (aux && aux->defined()) {
    TORCH_CHECK(aux->scalar_type() == at::kBFloat16 && aux->size(0) == M && aux->size(1) == N &&
                    aux->stride(1) == 1 && aux->stride(0) % 8 == 0 &&
                    (reinterpret_cast<uintptr_t>(aux->data_ptr()) & 15) == 0,
                "gemm: aux");
    auxt = *aux;
    args.aux_in = reinterpret_cast<const bf16*>(aux->data_ptr());
    args.ldx = aux->stride(0);
  }
  TORCH_CHECK((epi != EPI_GELU && epi != EPI_DGELU) || auxt.defined(), "gemm: gelu epilogues need aux");

  if (gather) {
    TORCH_CHECK(!a_trans && !b_trans && (epi == EPI_BF16 || epi == EPI_GELU || epi == EPI_LSE) && !accumulate,
                "gemm_gather: forward GEMMs (X @ W, bf16 / GELU / softmax-statistics epilogue) only");
    TORCH_CHECK(b.is_contiguous() && (K + kBK - 1) / kBK <= kGatherMaxKb, "gemm_gather: B must be contiguous, K <= 8192");
    args.g = *gather;
    args.g.local = reinterpret_cast<bf16*>(b.data_ptr());
    args.g.sub = (int)std::max<long>(1, std::min<long>(4096, ((long)kBK * N * 2 + 16383) / 16384));
  }
  // split-K is only wired for the fp32 / bf16 plain epilogues without bias or residual
  const bool can_split = !gather && ((epi == EPI_F32) || (epi == EPI_BF16 && !args.bias && !args.resid));
  int bn, splits;
  choose_tiling((int)M, (int)N, (int)K, bn, splits, can_split);
  // 2-SM 256x256 pair tiles whenever the 1-SM choice is 128x256 and M spans a pair
  // (force_bn: 128 / 256 pick a 1-SM width, 512 the 2-SM path)
  bool pair2 = (bn == 256 && M > 128);
  if (pair2) splits = choose_splits2((int)M, (int)N, (int)K, can_split);
  if (force_bn > 0) {
    pair2 = (force_bn == 512);
    bn = pair2 ? 256 : (int)force_bn;
  }
  if (force_splits > 0) splits = (int)force_splits;
  TORCH_CHECK(bn == 128 || bn == 256, "gemm: BN must be 128 or 256 (or 512 for the 2-SM path)");
  if (splits > 1 && !can_split) splits = 1;

  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  // A map: K-major [M rows, K cols] box {64, 128}; MN-major [K rows, M cols] box {64, 64}
  CUtensorMap ta = a_trans ? make_map(a.data_ptr(), K, M, a.stride(0), 64, 64)
                           : make_map(a.data_ptr(), M, K, a.stride(0), 64, kBM);
  CUtensorMap tb = b_trans ? make_map(b.data_ptr(), N, K, b.stride(0), 64, pair2 ? 128 : bn)
                           : make_map(b.data_ptr(), K, N, b.stride(0), 64, 64);

  GemmArgs run = args;
  torch::Tensor ws;
  CUtensorMap to, tx;
  if (splits > 1) {
    const long need = (long)splits * M * N;
    if (workspace && workspace->defined() && workspace->numel() >= need) {
      ws = *workspace;
    } else {
      ws = torch::empty({need}, a.options().dtype(at::kFloat));
    }
    run.epi = EPI_PARTIAL;
    run.splits = splits;
    to = make_store_map(ws.data_ptr(), true, M, N, N, splits);
  } else {
    run.splits = 1;
    to = make_store_map(out.data_ptr(), f32_out, M, N, out.stride(0));
  }
  if (epi == EPI_LSE) {
    const int tile_n = pair2 ? 256 : bn;
    const int np = 2 * (int)((N + tile_n - 1) / tile_n);
    *lse_part = torch::empty({M, np, 2}, a.options().dtype(at::kFloat));
    run.lse_part = reinterpret_cast<float2*>(lse_part->data_ptr<float>());
    run.lse_np = np;
  }
  tx = (epi == EPI_GELU) ? make_store_map(auxt.data_ptr(), false, M, N, auxt.stride(0)) : to;

#define DTB_GEMM_DISPATCH(BNV)                                                      \
  if (!a_trans && !b_trans) launch_gemm<BNV, false, true>(ta, tb, to, tx, run, st);   \
  else if (!a_trans && b_trans) launch_gemm<BNV, false, false>(ta, tb, to, tx, run, st); \
  else if (a_trans && !b_trans) launch_gemm<BNV, true, true>(ta, tb, to, tx, run, st);   \
  else launch_gemm<BNV, true, false>(ta, tb, to, tx, run, st);
  if (gather) {
    if (pair2) launch_gemm2<false, true, true>(ta, tb, to, tx, run, st);
    else if (bn == 256) launch_gemm<256, false, true, true>(ta, tb, to, tx, run, st);
    else launch_gemm<128, false, true, true>(ta, tb, to, tx, run, st);
  } else if (pair2) {
    if (!a_trans && !b_trans) launch_gemm2<false, true>(ta, tb, to, tx, run, st);
    else if (!a_trans && b_trans) launch_gemm2<false, false>(ta, tb, to, tx, run, st);
    else if (a_trans && !b_trans) launch_gemm2<true, true>(ta, tb, to, tx, run, st);
    else launch_gemm2<true, false>(ta, tb, to, tx, run, st);
  } else if (bn == 256) {
    DTB_GEMM_DISPATCH(256)
  } else {
    DTB_GEMM_DISPATCH(128)
  }
#undef DTB_GEMM_DISPATCH

  if (splits > 1) {
    const long MN = M * N;
    const int threads = 256;
    const long blocks = (MN / 4 + threads - 1) / threads;
    splitk_reduce_kernel<<<(unsigned)blocks, threads, 0, st>>>(
        reinterpret_cast<const float*>(ws.data_ptr()), splits, MN, (int)N,
        f32_out ? reinterpret_cast<float*>(out.data_ptr()) : nullptr,
        f32_out ? nullptr : reinterpret_cast<bf16*>(out.data_ptr()), out.stride(0), (float)alpha,
        accumulate ? 1 : 0);
    count_launch();
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

void gemm(torch::Tensor a, bool a_trans, torch::Tensor b, bool b_trans, torch::Tensor out, int64_t epi,
          c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> resid, c10::optional<torch::Tensor> aux,
          double alpha, bool accumulate, int64_t force_bn, int64_t force_splits,
          c10::optional<torch::Tensor> workspace) {
  gemm_impl(a, a_trans, b, b_trans, out, epi, bias, resid, aux, alpha, accumulate, force_bn, force_splits, workspace,
            nullptr);
}

// Forward GEMM out = X @ W (+ epilogue) with W's all-gather fused in: `b` is this
// rank's copy of W inside a flat bf16 buffer of `nflat` elements partitioned over
// `peers.size()` ranks (W starts at flat index `woff`; peers[r] is rank r's address
// of W[0][0], peer-mapped).  When state[GS_GEN] differs from state[GS_SITES + site]
// the kernel first pulls the other ranks' partitions of W into `b`, k-block by
// k-block, while the MMAs consume the k-blocks already in place; otherwise it is the
// plain GEMM.  All calls that share `state` must run on one stream.
// Returns the softmax partials for epi == EPI_LSE (see gemm_lse), else an undefined tensor.
torch::Tensor gemm_gather(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t epi,
                          c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> resid,
                          c10::optional<torch::Tensor> aux, std::vector<int64_t> peers, int64_t rank, int64_t woff,
                          int64_t nflat, torch::Tensor state, int64_t site) {
  const int W = (int)peers.size();
  TORCH_CHECK(W >= 1 && W <= kGatherRanks && rank >= 0 && rank < W, "gemm_gather: 1..8 ranks");
  TORCH_CHECK(state.is_cuda() && state.scalar_type() == at::kInt && state.is_contiguous() &&
                  state.numel() > GS_SITES + site && site >= 0,
              "gemm_gather: state must be an int32 CUDA tensor with room for the site");
  TORCH_CHECK(woff >= 0 && woff + b.numel() <= nflat, "gemm_gather: W outside the flat buffer");
  TORCH_CHECK(reinterpret_cast<int64_t>(b.data_ptr()) == peers[rank], "gemm_gather: peers[rank] must be b");
  GatherArgs g{};
  for (int r = 0; r < W; ++r) g.peer[r] = reinterpret_cast<const bf16*>(peers[r]);
  g.woff = woff;
  g.nflat = nflat;
  g.rank = (int)rank;
  g.world = W;
  g.site = (int)site;
  g.state = state.data_ptr<int>();
  torch::Tensor part;
  gemm_impl(a, false, b, false, out, epi, bias, resid, aux, 1.0, false, 0, 0, c10::nullopt, &g, &part);
  return part;
}

// LM head fused with the cross-entropy forward's reduction: out = X @ W (bf16) and,
// from the same epilogue, per row and column half-tile the (max, sum exp(x - max)) of
// the bf16-rounded outputs.  Returns the partials [M, np, 2]; xent_from_parts turns
// them into lse and the loss without reading the logits again.
torch::Tensor gemm_lse(torch::Tensor a, torch::Tensor b, torch::Tensor out) {
  torch::Tensor part;
  gemm_impl(a, false, b, false, out, EPI_LSE, c10::nullopt, c10::nullopt, c10::nullopt, 1.0, false, 0, 0,
            c10::nullopt, nullptr, &part);
  return part;
}

// Returns the (BN, splits) the heuristic would pick, for tests and tuning.
std::vector<int64_t> gemm_tiling(int64_t M, int64_t N, int64_t K) {
  int bn, s;
  choose_tiling((int)M, (int)N, (int)K, bn, s);
  return {bn, s};
}

DTB_DEFINE_STATUS_READER(status_gemm)

}  // namespace dtb
