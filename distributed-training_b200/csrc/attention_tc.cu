// Causal flash-attention forward on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Same contract as attn::fwd_kernel (attention.cu): reads q/k/v from the qkv GEMM
// output [B*T, 3*H*D] bf16, writes out [B*T, H*D] bf16 and the per-row
// log-sum-exp in the log2 domain (lse2 [B*H, T]) that the backward kernels use.
// Head dim 64.
//
// One CTA = one (batch*head, pair of 128-query tiles A and B); the two tiles share
// every K/V tile that both need.  10 warps:
//   warp 0      TMA: Q_A, Q_B once; K_j, V_j through a 2-stage ring (128 keys x 64).
//   warp 1      owns 512 TMEM columns (S_A, S_B: 128 each; O_A, O_B: 64 each); one
//               lane issues  S_t = Q_t K_j^T  (M=128, N=128, K=64) and
//               O_t += P_t V_j (M=128, N=64, K=128), committing to mbarriers.
//   warps 2..5  softmax for tile A, warps 6..9 for tile B: each thread owns one
//               query row, loads its 128 scores from TMEM, applies the causal mask,
//               keeps the running max / sum in registers (no shuffles), writes
//               P = exp2(s*scale*log2e - m) as bf16 into 128B-swizzled shared memory
//               (the K-major A operand of the PV MMA) and rescales its O row in
//               TMEM when the running max moved.
// While one tile's softmax runs, the MMA warp computes the other tile's scores, so
// tensor-core and SIMT/SFU work overlap.  All waits are bounded (common.cuh).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <mutex>

#include "common.cuh"

namespace dtb {
namespace attn_tc {

constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int D = 64;
constexpr int kThreads = 320;
constexpr int TILE = BQ * D * 2;         // 16 KB: one Q, K or V tile
constexpr int PBYTES = BQ * BKV * 2;     // 32 KB: one P tile (two 64-key swizzle atoms)
constexpr int STAGES = 2;
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + 2 * TILE;
constexpr int OFF_V = OFF_K + STAGES * TILE;
constexpr int OFF_P = OFF_V + STAGES * TILE;
constexpr int OFF_BAR = OFF_P + 2 * PBYTES;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
constexpr uint32_t TM_S = 0;    // S_t at column t*128
constexpr uint32_t TM_O = 256;  // O_t at column 256 + t*64

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2^x on the special-function unit (PTX ex2.approx; 2^-inf = +0).
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct Bars {
  uint64_t q_full;
  uint64_t k_full[STAGES], v_full[STAGES], kv_empty[STAGES];
  uint64_t s_full[2], s_free[2], p_full[2], o_done[2];
  uint32_t tmem_slot;
  int abort_flag;
};

// 320 threads, one CTA per SM.  10 warps put 3 warps on some schedulers, so the
// per-scheduler register file caps a thread at 168 registers.
__global__ void __launch_bounds__(kThreads, 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, bf16* __restrict__ out, float* __restrict__ lse2, int T,
                  int H, float sl2) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + OFF_BAR);
  volatile int* abort_flag = &bars->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int nq = (T + BQ - 1) / BQ;
  const int npairs = (nq + 1) / 2;
  const int pair = npairs - 1 - (int)blockIdx.x;  // heavy pairs first
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int C = H * D;
  const bool has_b = (2 * pair + 1) < nq;
  // tile t (0 = A, 1 = B) is query tile 2*pair + t; its last (diagonal) key tile has the same index
  const int n_kv = has_b ? 2 * pair + 2 : 2 * pair + 1;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->s_free[t], 4);
      mbar_init(&bars->p_full[t], 4);
      mbar_init(&bars->o_done[t], 1);
    }
    bars->abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQKV);
  }
  if (warp == 1) tmem_alloc(&bars->tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;
  const int row_base = b * T;  // first qkv row of this sequence

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- TMA
      mbar_arrive_expect_tx(&bars->q_full, (has_b ? 2 : 1) * TILE);
      tma_load_2d(&tmQKV, smem + OFF_Q, &bars->q_full, h * D, row_base + 2 * pair * BQ);
      if (has_b) tma_load_2d(&tmQKV, smem + OFF_Q + TILE, &bars->q_full, h * D, row_base + (2 * pair + 1) * BQ);
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        if (!mbar_wait(&bars->kv_empty[s], ph ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&bars->k_full[s], TILE);
        tma_load_2d(&tmQKV, smem + OFF_K + s * TILE, &bars->k_full[s], C + h * D, row_base + j * BKV);
        mbar_arrive_expect_tx(&bars->v_full[s], TILE);
        tma_load_2d(&tmQKV, smem + OFF_V + s * TILE, &bars->v_full[s], 2 * C + h * D, row_base + j * BKV);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA
      // Order: QK_A(0) QK_B(0) | PV_A(0) QK_A(1) | PV_B(0) QK_B(1) | PV_A(1) QK_A(2) | ...
      // Each tile's next scores are issued right after its PV, so the tensor core
      // works on one tile while the other tile's softmax runs.
      constexpr uint32_t id_qk = make_idesc_bf16(BQ, BKV, false, false);
      constexpr uint32_t id_pv = make_idesc_bf16(BQ, D, false, true);
      bool ok = mbar_wait(&bars->q_full, 0, abort_flag);
      auto issue_qk = [&](int t, int j) -> bool {
        const int s = j % STAGES;
        if (!mbar_wait(&bars->s_free[t], (j & 1) ^ 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t qbase = smem_u32(smem + OFF_Q + t * TILE);
        const uint32_t kbase = smem_u32(smem + OFF_K + s * TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma_f16(tmem + TM_S + t * 128, make_sw128_desc(qbase + kk * 32, 16, 1024),
                     make_sw128_desc(kbase + kk * 32, 16, 1024), id_qk, kk > 0 ? 1u : 0u);
        tc_commit(&bars->s_full[t]);
        return true;
      };
      if (ok) ok = mbar_wait(&bars->k_full[0], 0, abort_flag);
      if (ok) {
        tc_fence_after();
        ok = issue_qk(0, 0);
        if (ok && has_b) ok = issue_qk(1, 0);
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        if (!mbar_wait(&bars->v_full[s], ph, abort_flag)) { ok = false; break; }
        bool next_k_ready = false;
        const uint32_t vbase = smem_u32(smem + OFF_V + s * TILE);
        for (int t = 0; t < 2; ++t) {
          if (t == 1 && !has_b) continue;
          if (j > (2 * pair + t)) continue;
          if (!mbar_wait(&bars->p_full[t], j & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t pbase = smem_u32(smem + OFF_P + t * PBYTES);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)
            tc_mma_f16(tmem + TM_O + t * D, make_sw128_desc(pbase + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                       make_sw128_desc(vbase + kk * 2048, 8192, 1024), id_pv, (j > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&bars->o_done[t]);
          if (j + 1 <= (2 * pair + t)) {
            if (!next_k_ready) {
              const int s1 = (j + 1) % STAGES;
              if (!mbar_wait(&bars->k_full[s1], ((j + 1) / STAGES) & 1, abort_flag)) { ok = false; break; }
              tc_fence_after();
              next_k_ready = true;
            }
            if (!issue_qk(t, j + 1)) { ok = false; break; }
          }
        }
        if (!ok) break;
        tc_commit(&bars->kv_empty[s]);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax
    const int t = (warp - 2) >> 2;
    const int q = warp & 3;
    const bool active = (t == 0) || has_b;
    const int qtile = 2 * pair + t;
    const int r = q * 32 + lane;             // row within the tile (= TMEM lane)
    const int qrow = qtile * BQ + r;         // query index within the sequence
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    uint8_t* P = smem + OFF_P + t * PBYTES;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    if (active) {
      for (int j = 0; j <= (2 * pair + t) && ok; ++j) {
        if (!mbar_wait(&bars->s_full[t], j & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        uint32_t sr[128];
        tmem_ld32_issue(tmem + lane_off + TM_S + t * 128 + 0, sr);
        tmem_ld32_issue(tmem + lane_off + TM_S + t * 128 + 32, sr + 32);
        tmem_ld32_issue(tmem + lane_off + TM_S + t * 128 + 64, sr + 64);
        tmem_ld32_issue(tmem + lane_off + TM_S + t * 128 + 96, sr + 96);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->s_free[t]);
        // causal / length mask on the edge tiles, then the row max of the raw scores
        const int k0 = j * BKV;
        const bool edge = (j == (2 * pair + t)) || (k0 + BKV > T);
        if (edge) {
          const int lim = min(qrow + 1, T) - k0;  // keys [k0, k0+lim) are visible
#pragma unroll
          for (int c = 0; c < BKV; ++c)
            if (c >= lim) sr[c] = __float_as_uint(-INFINITY);
        }
        float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
        for (int c = 0; c < BKV; c += 4) {
          mx0 = fmaxf(mx0, __uint_as_float(sr[c]));
          mx1 = fmaxf(mx1, __uint_as_float(sr[c + 1]));
          mx2 = fmaxf(mx2, __uint_as_float(sr[c + 2]));
          mx3 = fmaxf(mx3, __uint_as_float(sr[c + 3]));
        }
        const float mcand = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl2;
        // Lazy rescaling: the reference max only moves when the new scores exceed it
        // by more than 2^8; P values stay <= 256, exact in the fp32 sum and fine in bf16.
        float alpha = 1.f;
        if (m == -INFINITY) {
          m = mcand;
        } else if (mcand > m + 8.f) {
          alpha = ex2_fast(m - mcand);
          m = mcand;
        }
        const float base = (m == -INFINITY) ? 0.f : m;
        float rs0 = 0.f, rs1 = 0.f, rs2 = 0.f, rs3 = 0.f;
#pragma unroll
        for (int c = 0; c < BKV; c += 4) {
          const float p0 = ex2_fast(fmaf(__uint_as_float(sr[c]), sl2, -base));
          const float p1 = ex2_fast(fmaf(__uint_as_float(sr[c + 1]), sl2, -base));
          const float p2 = ex2_fast(fmaf(__uint_as_float(sr[c + 2]), sl2, -base));
          const float p3 = ex2_fast(fmaf(__uint_as_float(sr[c + 3]), sl2, -base));
          sr[c] = __float_as_uint(p0);
          sr[c + 1] = __float_as_uint(p1);
          sr[c + 2] = __float_as_uint(p2);
          sr[c + 3] = __float_as_uint(p3);
          rs0 += p0;
          rs1 += p1;
          rs2 += p2;
          rs3 += p3;
        }
        l = l * alpha + ((rs0 + rs1) + (rs2 + rs3));
        // the previous PV must be done before P is overwritten and O rescaled
        if (j > 0 && !mbar_wait(&bars->o_done[t], (j - 1) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        // P row -> shared memory (K-major, 128B swizzle, two 64-key atoms)
#pragma unroll
        for (int ch = 0; ch < BKV / 8; ++ch) {
          const int atom = ch >> 3, k16 = ch & 7;
          uint4 u;
          u.x = pack_bf16x2(__uint_as_float(sr[ch * 8 + 0]), __uint_as_float(sr[ch * 8 + 1]));
          u.y = pack_bf16x2(__uint_as_float(sr[ch * 8 + 2]), __uint_as_float(sr[ch * 8 + 3]));
          u.z = pack_bf16x2(__uint_as_float(sr[ch * 8 + 4]), __uint_as_float(sr[ch * 8 + 5]));
          u.w = pack_bf16x2(__uint_as_float(sr[ch * 8 + 6]), __uint_as_float(sr[ch * 8 + 7]));
          *reinterpret_cast<uint4*>(P + atom * 16384 + r * 128 + ((k16 ^ (r & 7)) << 4)) = u;
        }
        // rescale this row of O when the running max moved (warp-uniform decision)
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t o[32];
            tmem_ld32_issue(tmem + lane_off + TM_O + t * D + half * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            tmem_st32(tmem + lane_off + TM_O + t * D + half * 32, o);
          }
          tmem_wait_st();
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full[t]);
      }
      // final: O / l
      if (ok && mbar_wait(&bars->o_done[t], (2 * pair + t) & 1, abort_flag)) {
        tc_fence_after();
        uint32_t o[64];
        tmem_ld32_issue(tmem + lane_off + TM_O + t * D, o);
        tmem_ld32_issue(tmem + lane_off + TM_O + t * D + 32, o + 32);
        tmem_wait_ld();
        if (qrow < T) {
          const float inv = l > 0.f ? 1.f / l : 0.f;
          bf16* orow = out + ((long)row_base + qrow) * C + h * D;
#pragma unroll
          for (int c = 0; c < 64; c += 8) {
            uint4 u;
            u.x = pack_bf16x2(__uint_as_float(o[c + 0]) * inv, __uint_as_float(o[c + 1]) * inv);
            u.y = pack_bf16x2(__uint_as_float(o[c + 2]) * inv, __uint_as_float(o[c + 3]) * inv);
            u.z = pack_bf16x2(__uint_as_float(o[c + 4]) * inv, __uint_as_float(o[c + 5]) * inv);
            u.w = pack_bf16x2(__uint_as_float(o[c + 6]) * inv, __uint_as_float(o[c + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c) = u;
          }
          lse2[(long)bh * T + qrow] = m + log2f(l);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// =============================================================================
// Backward.  Two deterministic kernels (no atomics), 6 warps each:
//   warp 0 TMA, warp 1 MMA (+ 256 TMEM columns), warps 2..5 element-wise math with
//   one 128-wide tile row per thread.  TMEM holds X (128 columns, reused for the
//   scores and then for dP) and the fp32 gradient accumulators.  Shared memory
//   (~97 KB) lets two CTAs share an SM, so one CTA's tensor work overlaps the
//   other's element-wise phase.
//
// dK/dV kernel: CTA = (batch*head, 128-key tile j); loops over query tiles i >= j:
//   X = K Q_i^T (S^T) -> P^T = exp2(S^T*scale*log2e - lse2[q])          (regs, bf16)
//   X = V dO_i^T (dP^T);  dV += P^T dO_i                                   (MMA)
//   dS^T = P^T * (dP^T - delta[q]);  dK += dS^T Q_i                         (MMA)
// dQ kernel: CTA = (batch*head, 128-query tile i); loops over key tiles j <= i:
//   X = Q K_j^T -> P;  X = dO V_j^T -> dS = P*(dP - delta);  dQ += dS K_j
// =============================================================================
constexpr int BW_THREADS = 192;
constexpr int BW_OFF_A = 0;                 // tile 0 (K for dkdv, Q for dq)
constexpr int BW_OFF_B = TILE;              // tile 1 (V for dkdv, dO for dq)
constexpr int BW_OFF_C = 2 * TILE;          // streamed tile (Q_i for dkdv, K_j for dq)
constexpr int BW_OFF_D = 3 * TILE;          // streamed tile (dO_i for dkdv, V_j for dq)
constexpr int BW_OFF_P = 4 * TILE;          // bf16 A operand: P^T then dS^T (dkdv), dS (dq)
constexpr int BW_OFF_LD = BW_OFF_P + PBYTES;  // [2][2][128] fp32 lse2 / delta (dkdv)
constexpr int BW_OFF_BAR = BW_OFF_LD + 2 * 2 * 128 * 4;
constexpr int BW_SMEM = BW_OFF_BAR + 256 + 1024;
constexpr uint32_t BW_X = 0, BW_G0 = 128, BW_G1 = 192;  // TMEM columns

struct BwBars {
  uint64_t fixed_full;                 // the two per-CTA tiles
  uint64_t c_full, c_empty, d_full, d_empty;
  uint64_t s_full, dp_full, ew_p, ew_ds, done;
  uint32_t tmem_slot;
  int abort_flag;
};

__device__ __forceinline__ void bw_init(BwBars* b) {
  mbar_init(&b->fixed_full, 1);
  mbar_init(&b->c_full, 1);
  mbar_init(&b->c_empty, 1);
  mbar_init(&b->d_full, 1);
  mbar_init(&b->d_empty, 1);
  mbar_init(&b->s_full, 1);
  mbar_init(&b->dp_full, 1);
  mbar_init(&b->ew_p, 4);
  mbar_init(&b->ew_ds, 4);
  mbar_init(&b->done, 1);
  b->abort_flag = 0;
  fence_barrier_init();
}

// Write 32 bf16-packed pairs (64 values) of this thread's row into the K-major
// 128B-swizzled A-operand tile at columns [c0, c0+64) (c0 multiple of 64).
__device__ __forceinline__ void put_row64(uint8_t* A, int r, int c0, const uint32_t* pk) {
  const int atom = c0 >> 6;
#pragma unroll
  for (int k16 = 0; k16 < 8; ++k16) {
    uint4 u = make_uint4(pk[k16 * 4 + 0], pk[k16 * 4 + 1], pk[k16 * 4 + 2], pk[k16 * 4 + 3]);
    *reinterpret_cast<uint4*>(A + atom * 16384 + r * 128 + ((k16 ^ (r & 7)) << 4)) = u;
  }
}

__device__ __forceinline__ float bf_lo(uint32_t p) { return __uint_as_float(p << 16); }
__device__ __forceinline__ float bf_hi(uint32_t p) { return __uint_as_float(p & 0xffff0000u); }

// Write 16 bf16-packed pairs (32 values) at columns [c0, c0+32) (c0 multiple of 32).
__device__ __forceinline__ void put_row32(uint8_t* A, int r, int c0, const uint32_t* pk) {
  const int atom = c0 >> 6, k0 = (c0 & 63) >> 3;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 u = make_uint4(pk[i * 4 + 0], pk[i * 4 + 1], pk[i * 4 + 2], pk[i * 4 + 3]);
    *reinterpret_cast<uint4*>(A + atom * 16384 + r * 128 + (((k0 + i) ^ (r & 7)) << 4)) = u;
  }
}

// Load 64 fp32 TMEM columns of this thread's row (every lane must call: the load
// is warp-collective) and, when `store` is set, write them scaled as bf16.
__device__ __forceinline__ void store_row64(uint32_t taddr, bf16* dst, float scale, bool store) {
  uint32_t o[64];
  tmem_ld32_issue(taddr, o);
  tmem_ld32_issue(taddr + 32, o + 32);
  tmem_wait_ld();
  if (!store) return;
#pragma unroll
  for (int c = 0; c < 64; c += 8) {
    uint4 u;
    u.x = pack_bf16x2(__uint_as_float(o[c + 0]) * scale, __uint_as_float(o[c + 1]) * scale);
    u.y = pack_bf16x2(__uint_as_float(o[c + 2]) * scale, __uint_as_float(o[c + 3]) * scale);
    u.z = pack_bf16x2(__uint_as_float(o[c + 4]) * scale, __uint_as_float(o[c + 5]) * scale);
    u.w = pack_bf16x2(__uint_as_float(o[c + 6]) * scale, __uint_as_float(o[c + 7]) * scale);
    *reinterpret_cast<uint4*>(dst + c) = u;
  }
}

template <bool DKDV>
__global__ void __launch_bounds__(BW_THREADS, 2)
    bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, const __grid_constant__ CUtensorMap tmDO,
                  const float* __restrict__ lse2, const float* __restrict__ delta, bf16* __restrict__ dqkv, int T,
                  int H, float sl2, float scale) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  BwBars* bars = reinterpret_cast<BwBars*>(smem + BW_OFF_BAR);
  volatile int* abort_flag = &bars->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = (T + 127) / 128;
  // dkdv: heavy (low) key tiles first; dq: heavy (high) query tiles first
  const int tile = DKDV ? (int)blockIdx.x : nt - 1 - (int)blockIdx.x;
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int C = H * D;
  const int row_base = b * T;
  const int it0 = DKDV ? tile : 0;            // streamed tile range
  const int it1 = DKDV ? nt - 1 : tile;
  const int n_it = it1 - it0 + 1;

  if (threadIdx.x == 0) {
    bw_init(bars);
    tma_prefetch_desc(&tmQKV);
    tma_prefetch_desc(&tmDO);
  }
  if (warp == 1) tmem_alloc(&bars->tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ TMA
      mbar_arrive_expect_tx(&bars->fixed_full, 2 * TILE);
      if (DKDV) {  // K_j, V_j
        tma_load_2d(&tmQKV, smem + BW_OFF_A, &bars->fixed_full, C + h * D, row_base + tile * 128);
        tma_load_2d(&tmQKV, smem + BW_OFF_B, &bars->fixed_full, 2 * C + h * D, row_base + tile * 128);
      } else {     // Q_i, dO_i
        tma_load_2d(&tmQKV, smem + BW_OFF_A, &bars->fixed_full, h * D, row_base + tile * 128);
        tma_load_2d(&tmDO, smem + BW_OFF_B, &bars->fixed_full, h * D, row_base + tile * 128);
      }
      for (int it = 0; it < n_it; ++it) {
        const int s = it0 + it;
        if (!mbar_wait(&bars->c_empty, (it & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&bars->c_full, TILE);
        if (DKDV) tma_load_2d(&tmQKV, smem + BW_OFF_C, &bars->c_full, h * D, row_base + s * 128);          // Q_i
        else tma_load_2d(&tmQKV, smem + BW_OFF_C, &bars->c_full, C + h * D, row_base + s * 128);           // K_j
        if (!mbar_wait(&bars->d_empty, (it & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&bars->d_full, TILE);
        if (DKDV) tma_load_2d(&tmDO, smem + BW_OFF_D, &bars->d_full, h * D, row_base + s * 128);           // dO_i
        else tma_load_2d(&tmQKV, smem + BW_OFF_D, &bars->d_full, 2 * C + h * D, row_base + s * 128);       // V_j
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA
      constexpr uint32_t id_s = make_idesc_bf16(128, 128, false, false);  // X = A0 * C^T  (both K-major)
      constexpr uint32_t id_g = make_idesc_bf16(128, D, false, true);     // G += P * (MN-major B)
      const uint32_t A0 = smem_u32(smem + BW_OFF_A), A1 = smem_u32(smem + BW_OFF_B);
      const uint32_t SC = smem_u32(smem + BW_OFF_C), SD = smem_u32(smem + BW_OFF_D);
      const uint32_t SP = smem_u32(smem + BW_OFF_P);
      bool ok = mbar_wait(&bars->fixed_full, 0, abort_flag);
      for (int it = 0; it < n_it && ok; ++it) {
        const uint32_t ph = it & 1;
        // X = A0 . C^T   (dkdv: K Q_i^T = S^T ; dq: Q K_j^T = S)
        if (!mbar_wait(&bars->c_full, ph, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma_f16(tmem + BW_X, make_sw128_desc(A0 + kk * 32, 16, 1024), make_sw128_desc(SC + kk * 32, 16, 1024),
                     id_s, kk > 0 ? 1u : 0u);
        tc_commit(&bars->s_full);
        // element-wise phase 1 done: X free, P (dkdv: P^T in smem) ready
        if (!mbar_wait(&bars->ew_p, ph, abort_flag)) { ok = false; break; }
        if (!mbar_wait(&bars->d_full, ph, abort_flag)) { ok = false; break; }
        tc_fence_after();
        // X = A1 . D^T   (dkdv: V dO_i^T = dP^T ; dq: dO V_j^T = dP)
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma_f16(tmem + BW_X, make_sw128_desc(A1 + kk * 32, 16, 1024), make_sw128_desc(SD + kk * 32, 16, 1024),
                     id_s, kk > 0 ? 1u : 0u);
        if (DKDV) {
          // dV += P^T . dO_i   (A = P^T smem, B = dO_i MN-major)
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            tc_mma_f16(tmem + BW_G1, make_sw128_desc(SP + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                       make_sw128_desc(SD + kk * 2048, 8192, 1024), id_g, (it > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&bars->dp_full);
        tc_commit(&bars->d_empty);
        if (!mbar_wait(&bars->ew_ds, ph, abort_flag)) { ok = false; break; }
        tc_fence_after();
        // dkdv: dK += dS^T . Q_i (B = Q_i MN-major);  dq: dQ += dS . K_j (B = K_j MN-major)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_f16(tmem + BW_G0, make_sw128_desc(SP + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                     make_sw128_desc(SC + kk * 2048, 8192, 1024), id_g, (it > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&bars->c_empty);
      }
      if (ok) tc_commit(&bars->done);
    }
  } else {
    // --------------------------------------------------------- element-wise
    const int q = warp & 3;
    const int r = q * 32 + lane;               // tile row (= TMEM lane)
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    uint8_t* A = smem + BW_OFF_P;
    float* LD = reinterpret_cast<float*>(smem + BW_OFF_LD);  // [slot][lse|delta][128]
    const float* lb = lse2 + (long)bh * T;
    const float* db = delta + (long)bh * T;
    const int my_row = tile * 128 + r;         // dkdv: key index; dq: query index
    float my_lse = 0.f, my_delta = 0.f;
    if (!DKDV && my_row < T) {
      my_lse = lb[my_row];
      my_delta = db[my_row];
    }
    bool ok = true;
    for (int it = 0; it < n_it && ok; ++it) {
      const uint32_t ph = it & 1;
      const int s = it0 + it;                  // streamed tile index
      float* Lsl = LD + (it & 1) * 256;
      if (DKDV) {
        const int qi = s * 128 + r;
        Lsl[r] = qi < T ? lb[qi] : 0.f;
        Lsl[128 + r] = qi < T ? db[qi] : 0.f;
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      // ---- phase 1: P (dkdv: P^T) from the scores
      if (!mbar_wait(&bars->s_full, ph, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t pk[64];  // this row's P as bf16 pairs
      // visibility: dkdv row = key kr, column = query qc: visible iff kr <= qc < T
      //             dq   row = query qr, column = key kc:   visible iff kc <= qr, kc < T
      const bool edge = (s == tile) || (s * 128 + 128 > T);
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t x[32];
        tmem_ld32_issue(tmem + lane_off + BW_X + ch * 32, x);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          float pv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int col = ch * 32 + c + e;
            const float lse_v = DKDV ? Lsl[col] : my_lse;
            float p = ex2_fast(fmaf(__uint_as_float(x[c + e]), sl2, -lse_v));
            if (edge) {
              const int gc = s * 128 + col;
              const bool vis = DKDV ? (gc >= my_row && gc < T) : (gc <= my_row && gc < T);
              if (!vis) p = 0.f;
            }
            pv[e] = p;
          }
          pk[ch * 16 + c / 2] = pack_bf16x2(pv[0], pv[1]);
        }
      }
      if (DKDV) {  // P^T is the A operand of dV += P^T dO
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) put_row32(A, r, ch * 32, pk + ch * 16);
        fence_proxy_async_smem();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->ew_p);
      // ---- phase 2: dS = P * (dP - delta)
      if (!mbar_wait(&bars->dp_full, ph, abort_flag)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t x[32], ds[16];
        tmem_ld32_issue(tmem + lane_off + BW_X + ch * 32, x);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const uint32_t pp = pk[ch * 16 + c / 2];
          const int col = ch * 32 + c;
          const float d0 = DKDV ? Lsl[128 + col] : my_delta;
          const float d1 = DKDV ? Lsl[128 + col + 1] : my_delta;
          ds[c / 2] = pack_bf16x2(bf_lo(pp) * (__uint_as_float(x[c]) - d0),
                                  bf_hi(pp) * (__uint_as_float(x[c + 1]) - d1));
        }
        put_row32(A, r, ch * 32, ds);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->ew_ds);
    }
    // ---- results
    if (ok && mbar_wait(&bars->done, 0, abort_flag)) {
      tc_fence_after();
      const bool st = my_row < T;
      const long ld = 3L * C;
      bf16* rowp = dqkv + ((long)row_base + (st ? my_row : 0)) * ld;
      if (DKDV) {
        store_row64(tmem + lane_off + BW_G0, rowp + C + h * D, scale, st);      // dK
        store_row64(tmem + lane_off + BW_G1, rowp + 2 * C + h * D, 1.f, st);    // dV
      } else {
        store_row64(tmem + lane_off + BW_G0, rowp + h * D, scale, st);          // dQ
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace attn_tc

typedef CUresult (*EncodeTiledFnA)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFnA encode_fn_attn() {
  static EncodeTiledFnA fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFnA>(p);
  });
  return fn;
}

// tcgen05 forward for head dim 64; writes out [B*T, H*64] and lse2 [B*H, T].
void attn_fwd_tc(torch::Tensor qkv, torch::Tensor out, torch::Tensor lse, int64_t B, int64_t T, int64_t H) {
  using namespace attn_tc;
  TORCH_CHECK(qkv.is_contiguous() && qkv.scalar_type() == at::kBFloat16 && qkv.numel() == B * T * 3 * H * D,
              "attn_fwd_tc: qkv must be contiguous bf16 [B*T, 3*H*64]");
  c10::cuda::CUDAGuard guard(qkv.device());
  bind_device_context(qkv.get_device());
  CUtensorMap m;
  const long rows = B * T, cols = 3 * H * D;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn_attn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, qkv.data_ptr(), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "attn_fwd_tc: tensor map encode failed ", (int)r);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    attr = true;
  }
  const int nq = (int)((T + BQ - 1) / BQ);
  dim3 grid((unsigned)((nq + 1) / 2), (unsigned)(B * H));
  const float sl2 = (float)(1.4426950408889634 / 8.0);  // log2(e) / sqrt(64)
  fwd_tc_kernel<<<grid, kThreads, SMEM_BYTES, at::cuda::getCurrentCUDAStream()>>>(
      m, reinterpret_cast<bf16*>(out.data_ptr()), lse.data_ptr<float>(), (int)T, (int)H, sl2);
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static CUtensorMap attn_map(const torch::Tensor& t, long rows, long cols) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn_attn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, t.data_ptr(), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "attention: tensor map encode failed ", (int)r);
  return m;
}

// tcgen05 backward for head dim 64: fills dqkv [B*T, 3*H*64] from qkv, dout
// [B*T, H*64], lse2 [B*H, T] and delta = rowsum(dout * out) [B*H, T].
void attn_bwd_tc(torch::Tensor qkv, torch::Tensor dout, torch::Tensor lse, torch::Tensor delta, torch::Tensor dqkv,
                 int64_t B, int64_t T, int64_t H) {
  using namespace attn_tc;
  TORCH_CHECK(dout.is_contiguous() && dout.numel() == B * T * H * D, "attn_bwd_tc: dout must be [B*T, H*64]");
  c10::cuda::CUDAGuard guard(qkv.device());
  bind_device_context(qkv.get_device());
  CUtensorMap mq = attn_map(qkv, B * T, 3 * H * D);
  CUtensorMap md = attn_map(dout, B * T, H * D);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(bwd_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, BW_SMEM);
    cudaFuncSetAttribute(bwd_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, BW_SMEM);
    attr = true;
  }
  const int nt = (int)((T + 127) / 128);
  dim3 grid((unsigned)nt, (unsigned)(B * H));
  const float scale = 0.125f;                               // 1/sqrt(64)
  const float sl2 = (float)(1.4426950408889634 / 8.0);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto* out = reinterpret_cast<bf16*>(dqkv.data_ptr());
  bwd_tc_kernel<true><<<grid, BW_THREADS, BW_SMEM, st>>>(mq, md, lse.data_ptr<float>(), delta.data_ptr<float>(), out,
                                                         (int)T, (int)H, sl2, scale);
  bwd_tc_kernel<false><<<grid, BW_THREADS, BW_SMEM, st>>>(mq, md, lse.data_ptr<float>(), delta.data_ptr<float>(),
                                                          out, (int)T, (int)H, sl2, scale);
  count_launch(2);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

DTB_DEFINE_STATUS_READER(status_attention_tc)

}  // namespace dtb
