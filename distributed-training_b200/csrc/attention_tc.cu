// Causal flash-attention forward on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Same contract as attn::fwd_kernel (attention.cu): reads q/k/v from the qkv GEMM
// output [B*T, 3*H*D] bf16, writes out [B*T, H*D] bf16 and the per-row
// log-sum-exp in the log2 domain (lse2 [B*H, T]) that the backward kernels use.
// Head dim 64.
//
// One CTA = one (batch*head, pair of 128-query tiles A and B); the two tiles share
// every K/V tile that both need.  10 warps:
//   warp 0      TMA: Q_A, Q_B once; K_j, V_j through 3-stage rings (128 keys x 64).
//   warp 1      owns 512 TMEM columns (S_A, S_B: 128 each; O_A, O_B: 64 each; bf16
//               P_A, P_B: 64 each); one lane issues  S_t = Q_t K_j^T  (M=128, N=128,
//               K=64, both operands in shared memory) and O_t += P_t V_j (M=128,
//               N=64, K=128, A = P_t read from TMEM), committing to mbarriers.
//   warps 2..5  softmax for tile A, warps 6..9 for tile B: each thread owns one
//               query row, loads its 128 scores from TMEM, applies the causal mask,
//               keeps the running max / sum in registers (no shuffles), writes
//               P = exp2(s*scale*log2e - m) as bf16 into its own TMEM lane (the A
//               operand of the PV MMA, so P never touches shared memory) and
//               rescales its O row in TMEM when the running max moved.
// A tile's next scores S_t(j+1) are computed while its softmax of step j runs (the
// scores are copied to registers first), and its PV runs while the softmax of
// step j+1 computes exponentials, so the softmax warps run back to back and the
// tensor core hides behind them.  All waits are bounded (common.cuh).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <mutex>

#include <cstdlib>
#include <string>

#include "common.cuh"

namespace dtb {
namespace attn_tc {

constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int D = 64;
constexpr int kThreads = 320;
constexpr int TILE = BQ * D * 2;         // 16 KB: one Q, K or V tile
constexpr int PBYTES = BQ * BKV * 2;     // 32 KB: one P tile (two 64-key swizzle atoms)
constexpr int STAGES = 3;
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + 2 * TILE;
constexpr int OFF_V = OFF_K + STAGES * TILE;
constexpr int OFF_BAR = OFF_V + STAGES * TILE;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
constexpr uint32_t TM_S = 0;    // S_t at column t*128
constexpr uint32_t TM_O = 256;  // O_t at column 256 + t*64
constexpr uint32_t TM_P = 384;  // bf16 P_t (64 packed columns) at 384 + t*64: the A operand of O += P V

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
__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// 2^x on the special-function unit (PTX ex2.approx; 2^-inf = +0).
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}


// ---------------------------------------------------------------- softmax math
// Packed-FP32 (f32x2) and 3-input max instructions of sm_100: one instruction
// does two FMAs / adds, or folds two values into a running max.
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// (a0, a1) = (a0, a1) * (b0, b1) + (c0, c1)
__device__ __forceinline__ void ffma2(float& a0, float& a1, float b0, float b1, float c0, float c1) {
  asm("{\n\t.reg .b64 xa, xb, xc;\n\t"
      "mov.b64 xa, {%0, %1};\n\tmov.b64 xb, {%2, %3};\n\tmov.b64 xc, {%4, %5};\n\t"
      "fma.rn.f32x2 xa, xa, xb, xc;\n\tmov.b64 {%0, %1}, xa;\n\t}"
      : "+f"(a0), "+f"(a1) : "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
// (a0, a1) += (b0, b1)
__device__ __forceinline__ void fadd2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 xa, xb;\n\t"
      "mov.b64 xa, {%0, %1};\n\tmov.b64 xb, {%2, %3};\n\t"
      "add.rn.f32x2 xa, xa, xb;\n\tmov.b64 {%0, %1}, xa;\n\t}"
      : "+f"(a0), "+f"(a1) : "f"(b0), "f"(b1));
}
// (a0, a1) -= (b0, b1)
__device__ __forceinline__ void fsub2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 xa, xb;\n\t"
      "mov.b64 xa, {%0, %1};\n\tmov.b64 xb, {%2, %3};\n\t"
      "sub.rn.f32x2 xa, xa, xb;\n\tmov.b64 {%0, %1}, xa;\n\t}"
      : "+f"(a0), "+f"(a1) : "f"(b0), "f"(b1));
}
// The softmax uses ex2 (special-function unit) and cvt-based bf16 packing.  Measured
// on B200 (B=16, T=1024, H=12): with exponentials, packing and stores fused in one
// pass this is faster than moving part of the exponentials to a polynomial on the
// FMA pipe (1/4 of them: 98 vs 94 us; 1/2: 105 us) or packing on the integer pipe.

struct Bars {
  uint64_t q_full;
  uint64_t k_full[STAGES], v_full[STAGES], k_empty[STAGES], v_empty[STAGES];
  uint64_t s_full[2], s_free[2], p_full[2], o_done[2];
  uint32_t tmem_slot;
  int abort_flag;
};

// 320 threads, one CTA per SM.  10 warps put 3 warps on some schedulers, so the
// per-scheduler register file caps a thread at 168 registers.
__global__ void __maxnreg__(DTB_CORESIDENT_MAXNREG_ATTN)
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
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_empty[s], 1);
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
        // K and V stages are released separately: K_j once its scores are computed,
        // V_j once its PV products are, so the next keys stream in early
        if (!mbar_wait(&bars->k_empty[s], ph ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&bars->k_full[s], TILE);
        tma_load_2d(&tmQKV, smem + OFF_K + s * TILE, &bars->k_full[s], C + h * D, row_base + j * BKV);
        if (!mbar_wait(&bars->v_empty[s], ph ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&bars->v_full[s], TILE);
        tma_load_2d(&tmQKV, smem + OFF_V + s * TILE, &bars->v_full[s], 2 * C + h * D, row_base + j * BKV);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA
      // Per key tile j:  QK_A(j+1) QK_B(j+1) | PV_A(j) PV_B(j).
      // A tile's next scores are issued as soon as its softmax has copied the
      // current scores out of TMEM (s_free), so they are ready when that softmax
      // finishes and the softmax warps never wait on the tensor core for scores.
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
        if (ok) tc_commit(&bars->k_empty[0]);
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        // next scores of every tile that still has key tile j+1
        if (j + 1 < n_kv) {
          const int s1 = (j + 1) % STAGES;
          if (!mbar_wait(&bars->k_full[s1], ((j + 1) / STAGES) & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          for (int t = 0; t < 2 && ok; ++t) {
            if (t == 1 && !has_b) continue;
            if (j + 1 > (2 * pair + t)) continue;
            ok = issue_qk(t, j + 1);
          }
          if (!ok) break;
          tc_commit(&bars->k_empty[s1]);
        }
        if (!mbar_wait(&bars->v_full[s], ph, abort_flag)) { ok = false; break; }
        const uint32_t vbase = smem_u32(smem + OFF_V + s * TILE);
        for (int t = 0; t < 2; ++t) {
          if (t == 1 && !has_b) continue;
          if (j > (2 * pair + t)) continue;
          if (!mbar_wait(&bars->p_full[t], j & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)  // A = P_t from TMEM, 8 packed columns per K=16 slice
            tc_mma_f16_ts(tmem + TM_O + t * D, tmem + TM_P + t * 64 + kk * 8,
                          make_sw128_desc(vbase + kk * 2048, 8192, 1024), id_pv, (j > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&bars->o_done[t]);
        }
        if (!ok) break;
        tc_commit(&bars->v_empty[s]);
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
        for (int c = 0; c < BKV; c += 8) {
          mx0 = max3f(mx0, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
          mx1 = max3f(mx1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
          mx2 = max3f(mx2, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
          mx3 = max3f(mx3, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
        }
        const float mcand = fmaxf(max3f(mx0, mx1, mx2), mx3) * sl2;
        // Lazy rescaling: the reference max only moves when the new scores exceed it
        // by more than 2^8; P values stay <= 256, exact in the fp32 sum and fine in bf16.
        float alpha = 1.f;
        if (m == -INFINITY) {
          m = mcand;
        } else if (mcand > m + 8.f) {
          alpha = ex2_fast(m - mcand);
          m = mcand;
        }
        const float nb = (m == -INFINITY) ? 0.f : -m;
        // the previous PV must be done before P is overwritten and O rescaled; it was
        // issued when this tile's previous P was published, so this rarely waits
        if (j > 0 && !mbar_wait(&bars->o_done[t], (j - 1) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        // exponentials, row sum and the bf16 P row (into this thread's TMEM lane, the A
        // operand of the PV product) in one pass of 8-column chunks, so the
        // special-function unit (ex2), the packing and the TMEM stores run concurrently
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
        for (int ch = 0; ch < BKV / 8; ++ch) {
          float x[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] = __uint_as_float(sr[ch * 8 + e]);
#pragma unroll
          for (int e = 0; e < 8; e += 2) ffma2(x[e], x[e + 1], sl2, sl2, nb, nb);
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] = ex2_fast(x[e]);
          fadd2(s0, s1, x[0], x[1]);
          fadd2(s2, s3, x[2], x[3]);
          fadd2(s0, s1, x[4], x[5]);
          fadd2(s2, s3, x[6], x[7]);
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w[e] = pack_bf16x2(x[2 * e], x[2 * e + 1]);
          tmem_st4(tmem + lane_off + TM_P + t * 64 + ch * 4, w[0], w[1], w[2], w[3]);
        }
        l = l * alpha + ((s0 + s1) + (s2 + s3));
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
        }
        tmem_wait_st();  // P (and a rescaled O) are in TMEM before the PV product is released
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
// Backward.  Two deterministic kernels (no atomics) with the forward's layout:
// 10 warps, one CTA per SM, two 128-row sub-tiles A and B per CTA whose tensor
// work and element-wise work interleave (while one sub-tile's warps compute
// exponentials, the tensor core runs the other's products).
//   warp 0      TMA: the four fixed tiles, then the streamed tiles through
//               2-stage rings (one ring per streamed operand).
//   warp 1      owns 512 TMEM columns: X_t (128, scores and then dP) and the fp32
//               gradient accumulators; one lane issues every tcgen05.mma.
//   warps 2..5  element-wise math of sub-tile A, warps 6..9 of sub-tile B: one
//               query row per thread (the TMEM lane), so lse and delta are scalars.
//
// dK/dV kernel: CTA = (batch*head, pair of 128-key tiles kA=2p, kB=2p+1); loops
// over query tiles i >= kA (sub-tile B starts at i = kB):
//   X_t = Q_i K_t^T -> P = exp2(S*scale*log2e - lse2[q])  (regs; bf16 P -> smem)
//   X_t = dO_i V_t^T (dP);  dV_t += P^T dO_i   (A = P read MN-major)
//   dS = P * (dP - delta[q])  (bf16 -> smem);  dK_t += dS^T Q_i
// dQ kernel: CTA = (batch*head, pair of 128-query tiles), loops over key tiles j:
//   X_t = Q_t K_j^T -> P;  X_t = dO_t V_j^T -> dS = P*(dP - delta);  dQ_t += dS K_j
// Reference math: dtrain/autograd.py:226-252 (attention backward).
// =============================================================================
constexpr int BW_THREADS = 320;
constexpr int BW_OFF_F = 0;                     // fixed tiles [t][2]: dkdv K_t, V_t; dq Q_t, dO_t
constexpr int BW_OFF_S0 = 4 * TILE;             // streamed ring 0 [2]: dkdv Q_i; dq K_j
constexpr int BW_OFF_S1 = 6 * TILE;             // streamed ring 1 [2]: dkdv dO_i; dq V_j
constexpr int BW_OFF_P = 8 * TILE;              // [t] bf16 P then dS (128 query rows x 128 keys)
constexpr int BW_OFF_BAR = BW_OFF_P + 2 * PBYTES;
constexpr int BW_SMEM = BW_OFF_BAR + 512 + 1024;
constexpr uint32_t BW_X = 0, BW_G = 256;        // X_t at t*128; G0_t at 256 + t*128, G1_t at 256 + t*128 + 64
constexpr uint32_t BW_DS = 64;                   // dq: bf16 dS_t (64 packed columns) at 256 + t*128 + 64

struct BwBars {
  uint64_t fixed_full;
  uint64_t s0_full[2], s0_empty[2], s1_full[2], s1_empty[2];
  uint64_t s_full[2], x_free[2], p_ready[2], dp_full[2], pv_done[2], x_free2[2], ds_ready[2], ds_done[2];
  uint64_t ds_free[2];  // dK/dV with dS stores: the store of sub-tile t's dS tile has read it
  uint64_t done;
  uint32_t tmem_slot;
  int abort_flag;
};

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

__device__ __forceinline__ float bf_lo(uint32_t p) { return __uint_as_float(p << 16); }
__device__ __forceinline__ float bf_hi(uint32_t p) { return __uint_as_float(p & 0xffff0000u); }

// Write this thread's 128-key bf16 row (64 packed words) into a [128 rows][128 keys]
// tile laid out as two 128B-swizzled 64-key atoms: the K-major A operand of dQ
// (M = queries) and, read with the MN-major descriptor, the A operand P^T / dS^T
// of dV / dK (M = keys).
__device__ __forceinline__ void put_row128(uint8_t* A, int r, const uint32_t* pk) {
#pragma unroll
  for (int ch = 0; ch < 16; ++ch) {
    const int atom = ch >> 3, k16 = ch & 7;
    *reinterpret_cast<uint4*>(A + atom * 16384 + r * 128 + ((k16 ^ (r & 7)) << 4)) =
        make_uint4(pk[ch * 4 + 0], pk[ch * 4 + 1], pk[ch * 4 + 2], pk[ch * 4 + 3]);
  }
}

template <bool DKDV>
__global__ void __maxnreg__(DTB_CORESIDENT_MAXNREG_ATTN)
    bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, const __grid_constant__ CUtensorMap tmDO,
                  const __grid_constant__ CUtensorMap tmDS, const float* __restrict__ lse2, float* __restrict__ delta,
                  const bf16* __restrict__ out, const bf16* __restrict__ dout, bf16* __restrict__ dqkv, int T, int H,
                  float sl2, float scale, int store_ds) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  BwBars* bars = reinterpret_cast<BwBars*>(smem + BW_OFF_BAR);
  volatile int* abort_flag = &bars->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = (T + 127) / 128;
  const int npairs = (nt + 1) / 2;
  // dkdv: low key pairs have the most query tiles; dq: high query pairs the most key tiles
  const int pair = DKDV ? (int)blockIdx.x : npairs - 1 - (int)blockIdx.x;
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int C = H * D;
  const int row_base = b * T;
  const bool has_b = 2 * pair + 1 < nt;
  // streamed tile range [s_lo, s_hi]; sub-tile t is active for s in [lo_t, hi_t]
  const int s_lo = DKDV ? 2 * pair : 0;
  const int s_hi = DKDV ? nt - 1 : (has_b ? 2 * pair + 1 : 2 * pair);
  auto lo_of = [&](int t) { return DKDV ? 2 * pair + t : 0; };
  auto hi_of = [&](int t) { return DKDV ? nt - 1 : 2 * pair + t; };
  auto active = [&](int t, int s) { return (t == 0 || has_b) && s >= lo_of(t) && s <= hi_of(t); };

  if (threadIdx.x == 0) {
    mbar_init(&bars->fixed_full, 1);
    for (int k = 0; k < 2; ++k) {
      mbar_init(&bars->s0_full[k], 1);
      mbar_init(&bars->s0_empty[k], 1);
      mbar_init(&bars->s1_full[k], 1);
      mbar_init(&bars->s1_empty[k], 1);
      mbar_init(&bars->s_full[k], 1);
      mbar_init(&bars->x_free[k], 4);
      mbar_init(&bars->p_ready[k], 4);
      mbar_init(&bars->dp_full[k], 1);
      mbar_init(&bars->pv_done[k], 1);
      mbar_init(&bars->x_free2[k], 4);
      mbar_init(&bars->ds_ready[k], 4);
      mbar_init(&bars->ds_done[k], 1);
      mbar_init(&bars->ds_free[k], 1);
    }
    mbar_init(&bars->done, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQKV);
    tma_prefetch_desc(&tmDO);
    if (DKDV && store_ds) tma_prefetch_desc(&tmDS);
  }
  if (warp == 1) tmem_alloc(&bars->tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ TMA
      const int nfixed = has_b ? 2 : 1;
      mbar_arrive_expect_tx(&bars->fixed_full, nfixed * 2 * TILE);
      for (int t = 0; t < nfixed; ++t) {
        const int row = row_base + (2 * pair + t) * 128;
        uint8_t* f = smem + BW_OFF_F + t * 2 * TILE;
        if (DKDV) {  // K_t, V_t
          tma_load_2d(&tmQKV, f, &bars->fixed_full, C + h * D, row);
          tma_load_2d(&tmQKV, f + TILE, &bars->fixed_full, 2 * C + h * D, row);
        } else {     // Q_t, dO_t
          tma_load_2d(&tmQKV, f, &bars->fixed_full, h * D, row);
          tma_load_2d(&tmDO, f + TILE, &bars->fixed_full, h * D, row);
        }
      }
      for (int s = s_lo; s <= s_hi; ++s) {
        const int it = s - s_lo, st = it & 1;
        const uint32_t ph = ((it >> 1) & 1) ^ 1;
        const int row = row_base + s * 128;
        if (!mbar_wait(&bars->s0_empty[st], ph, abort_flag)) break;
        mbar_arrive_expect_tx(&bars->s0_full[st], TILE);
        if (DKDV) tma_load_2d(&tmQKV, smem + BW_OFF_S0 + st * TILE, &bars->s0_full[st], h * D, row);       // Q_i
        else tma_load_2d(&tmQKV, smem + BW_OFF_S0 + st * TILE, &bars->s0_full[st], C + h * D, row);        // K_j
        if (!mbar_wait(&bars->s1_empty[st], ph, abort_flag)) break;
        mbar_arrive_expect_tx(&bars->s1_full[st], TILE);
        if (DKDV) tma_load_2d(&tmDO, smem + BW_OFF_S1 + st * TILE, &bars->s1_full[st], h * D, row);        // dO_i
        else tma_load_2d(&tmQKV, smem + BW_OFF_S1 + st * TILE, &bars->s1_full[st], 2 * C + h * D, row);   // V_j
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA
      constexpr uint32_t id_s = make_idesc_bf16(128, 128, false, false);           // X = A . B^T, both K-major
      constexpr uint32_t id_g = make_idesc_bf16(128, D, DKDV, true);                // G += P(^T) . (MN-major B)
      const uint32_t F = smem_u32(smem + BW_OFF_F);
      const uint32_t S0 = smem_u32(smem + BW_OFF_S0), S1 = smem_u32(smem + BW_OFF_S1);
      const uint32_t SP = smem_u32(smem + BW_OFF_P);
      // X_t = (dkdv) streamed . fixed^T  /  (dq) fixed . streamed^T   (M = queries)
      auto issue_x = [&](int t, uint32_t fixed_tile, uint32_t streamed_tile) {
        const uint32_t a = DKDV ? streamed_tile : fixed_tile, bb = DKDV ? fixed_tile : streamed_tile;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma_f16(tmem + BW_X + t * 128, make_sw128_desc(a + kk * 32, 16, 1024),
                     make_sw128_desc(bb + kk * 32, 16, 1024), id_s, kk > 0 ? 1u : 0u);
      };
      // G_t(col) += A(P or dS of sub-tile t) . B (streamed tile, MN-major)
      auto issue_g = [&](int t, uint32_t col, uint32_t btile, bool acc) {
        const uint32_t pa = SP + t * PBYTES;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t bd = make_sw128_desc(btile + kk * 2048, 8192, 1024);
          if (DKDV)  // A = P^T / dS^T, read MN-major from shared memory
            tc_mma_f16(tmem + col, make_sw128_desc(pa + kk * 2048, 16384, 1024), bd, id_g, (acc || kk > 0) ? 1u : 0u);
          else       // A = dS from tensor memory (BW_DS columns of sub-tile t)
            tc_mma_f16_ts(tmem + col, tmem + BW_G + t * 128 + BW_DS + kk * 8, bd, id_g, (acc || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(&bars->fixed_full, 0, abort_flag);
      if (ok) ok = mbar_wait(&bars->s0_full[0], 0, abort_flag);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < 2; ++t)
          if (active(t, s_lo)) {
            issue_x(t, F + t * 2 * TILE, S0);
            tc_commit(&bars->s_full[t]);
          }
      }
      // dS tile stores issued in the previous iteration have long read their source by
      // the next one: confirm that there and release the tiles (ds_free) to the
      // element-wise warps, which write the next P into them - so waiting for a store
      // never holds up the MMA issue
      bool store_pending[2] = {false, false};
      auto release_stored = [&]() {
        if (!(store_pending[0] || store_pending[1])) return;
        bulk_wait_read0();
        for (int t = 0; t < 2; ++t)
          if (store_pending[t]) {
            mbar_arrive(&bars->ds_free[t]);
            store_pending[t] = false;
          }
      };
      for (int s = s_lo; s <= s_hi && ok; ++s) {
        const int it = s - s_lo, st = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        const uint32_t s0 = S0 + st * TILE, s1 = S1 + st * TILE;
        if (DKDV && store_ds) release_stored();
        if (!mbar_wait(&bars->s1_full[st], ph, abort_flag)) { ok = false; break; }
        // dP_t = dO . V^T into X_t once the element-wise warps have read the scores
        for (int t = 0; t < 2 && ok; ++t) {
          if (!active(t, s)) continue;
          const uint32_t k = (uint32_t)(s - lo_of(t));
          if (!mbar_wait(&bars->x_free[t], k & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          issue_x(t, F + t * 2 * TILE + TILE, s1);
          tc_commit(&bars->dp_full[t]);
        }
        if (!ok) break;
        if (DKDV) {  // dV_t += P^T dO_i
          for (int t = 0; t < 2 && ok; ++t) {
            if (!active(t, s)) continue;
            const uint32_t k = (uint32_t)(s - lo_of(t));
            if (!mbar_wait(&bars->p_ready[t], k & 1, abort_flag)) { ok = false; break; }
            tc_fence_after();
            issue_g(t, BW_G + t * 128 + 64, s1, k > 0);
            tc_commit(&bars->pv_done[t]);
          }
          if (!ok) break;
        }
        tc_commit(&bars->s1_empty[st]);
        // Per sub-tile: its next scores as soon as dP has been read out of X_t (x_free2),
        // then dK_t += dS^T Q_i / dQ_t += dS K_j once dS is in shared memory.  The
        // element-wise warps find the next scores ready when they finish storing dS.
        bool next_ready = false;
        for (int t = 0; t < 2 && ok; ++t) {
          const bool act = active(t, s);
          const uint32_t k = act ? (uint32_t)(s - lo_of(t)) : 0u;
          if (s + 1 <= s_hi && active(t, s + 1)) {
            const int st1 = (it + 1) & 1;
            if (!next_ready) {
              if (!mbar_wait(&bars->s0_full[st1], ((it + 1) >> 1) & 1, abort_flag)) { ok = false; break; }
              next_ready = true;
            }
            if (act && !mbar_wait(&bars->x_free2[t], k & 1, abort_flag)) { ok = false; break; }
            tc_fence_after();
            issue_x(t, F + t * 2 * TILE, S0 + st1 * TILE);
            tc_commit(&bars->s_full[t]);
          }
          if (act) {
            if (!mbar_wait(&bars->ds_ready[t], k & 1, abort_flag)) { ok = false; break; }
            tc_fence_after();
            if (DKDV && store_ds) {
              // dS tile (queries of tile s x the sub-tile's 128 keys) -> global, for the dQ GEMM
              const uint8_t* ds = smem + BW_OFF_P + t * PBYTES;
              tma_store_3d(&tmDS, ds, (2 * pair + t) * 128, s * 128, bh);
              tma_store_3d(&tmDS, ds + 16384, (2 * pair + t) * 128 + 64, s * 128, bh);
              bulk_commit();
            }
            issue_g(t, BW_G + t * 128, s0, k > 0);
            tc_commit(&bars->ds_done[t]);
            if (DKDV && store_ds) store_pending[t] = true;  // released at the top of the next iteration
          }
        }
        if (!ok) break;
        tc_commit(&bars->s0_empty[st]);
      }
      if (ok) tc_commit(&bars->done);
      if (DKDV && store_ds) bulk_wait0();  // the dS stores are complete before the kernel ends
    }
  } else {
    // --------------------------------------------------------- element-wise
    const int t = (warp - 2) >> 2;
    const int q = warp & 3;
    const int r = q * 32 + lane;                     // tile row = query row = TMEM lane
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    uint8_t* A = smem + BW_OFF_P + t * PBYTES;
    const float* lb = lse2 + (long)bh * T;
    const float* db = delta + (long)bh * T;
    const uint32_t xcol = BW_X + t * 128;
    (void)db;
    bool ok = true;
    if (t == 0 || has_b) {
      const int lo = lo_of(t), hi = hi_of(t);
      // lse / delta of this thread's query row; dkdv rows change with the streamed tile
      float my_lse = 0.f, my_delta = 0.f;
      auto load_ld = [&](int qi, float& l, float& d) {
        l = qi < T ? lb[qi] : 0.f;
        d = qi < T ? db[qi] : 0.f;
      };
      if (DKDV) {
        load_ld(lo * 128 + r, my_lse, my_delta);
      } else {
        // The dQ kernel runs first and produces delta = rowsum(dO * O) for its own
        // query rows (fp32 sum of the bf16 products, 64 terms in order); the dK/dV
        // kernel reads it afterwards.
        const int qi = (2 * pair + t) * 128 + r;
        my_lse = qi < T ? lb[qi] : 0.f;
        if (qi < T) {
          const long off = ((long)row_base + qi) * C + h * D;
          const uint4* op = reinterpret_cast<const uint4*>(out + off);
          const uint4* gp = reinterpret_cast<const uint4*>(dout + off);
          float acc = 0.f;
#pragma unroll
          for (int v = 0; v < D / 8; ++v) {
            const uint4 a = op[v], g = gp[v];
            const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, gw[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              acc = fmaf(bf_lo(aw[e]), bf_lo(gw[e]), acc);
              acc = fmaf(bf_hi(aw[e]), bf_hi(gw[e]), acc);
            }
          }
          my_delta = acc;
          delta[(long)bh * T + qi] = acc;
        }
      }
      for (int s = lo; s <= hi && ok; ++s) {
        const uint32_t k = (uint32_t)(s - lo);
        const int qrow = (DKDV ? s : 2 * pair + t) * 128 + r;   // query index within the sequence
        const int kbase = (DKDV ? 2 * pair + t : s) * 128;       // first key of the tile
        float nl = 0.f, nd = 0.f;
        if (DKDV && s < hi) load_ld(qrow + 128, nl, nd);        // prefetch the next rows' statistics
        // ---- phase 1: P = exp2(S*scale*log2e - lse)
        if (!mbar_wait(&bars->s_full[t], k & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        // keys [kbase, kbase + lim) are visible to this query (none for rows past T)
        const int lim = qrow < T ? min(qrow + 1, T) - kbase : 0;
        const bool need_mask = __any_sync(0xffffffffu, lim < 128);
        const float nb = -my_lse;
        uint32_t pk[64];
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {  // 32 columns per TMEM load keeps P + one chunk in registers
          uint32_t x[32];
          tmem_ld32_issue(tmem + lane_off + xcol + ch * 32, x);
          tmem_wait_ld();
          if (ch == 3) {  // scores read: X_t may take dP
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->x_free[t]);
          }
          if (need_mask) {
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (ch * 32 + c >= lim) x[c] = __float_as_uint(-INFINITY);
          }
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            float p0 = __uint_as_float(x[c]), p1 = __uint_as_float(x[c + 1]);
            ffma2(p0, p1, sl2, sl2, nb, nb);
            pk[ch * 16 + (c >> 1)] = pack_bf16x2(ex2_fast(p0), ex2_fast(p1));
          }
        }
        if (DKDV) {  // P is the A operand of dV += P^T dO: the previous dS must have been consumed
          if (k > 0 && !mbar_wait(&bars->ds_done[t], (k - 1) & 1, abort_flag)) { ok = false; break; }
          // ... and, when it is stored for the dQ GEMM, read by its store
          if (k > 0 && store_ds && !mbar_wait(&bars->ds_free[t], (k - 1) & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          put_row128(A, r, pk);
          fence_proxy_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->p_ready[t]);
        }
        // ---- phase 2: dS = P * (dP - delta), in place over the packed P
        if (!mbar_wait(&bars->dp_full[t], k & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t x[32];
          tmem_ld32_issue(tmem + lane_off + xcol + ch * 32, x);
          tmem_wait_ld();
          if (ch == 3) {  // dP read: X_t may take the next scores
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->x_free2[t]);
          }
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const uint32_t pp = pk[ch * 16 + c / 2];
            float d0 = __uint_as_float(x[c]), d1 = __uint_as_float(x[c + 1]);
            fsub2(d0, d1, my_delta, my_delta);
            pk[ch * 16 + c / 2] = pack_bf16x2(bf_lo(pp) * d0, bf_hi(pp) * d1);
          }
        }
        // the dS tile overwrites P: dkdv waits for dV (P^T dO), dq for the previous dQ
        if (DKDV) {
          if (!mbar_wait(&bars->pv_done[t], k & 1, abort_flag)) { ok = false; break; }
        } else if (k > 0 && !mbar_wait(&bars->ds_done[t], (k - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (DKDV) {
          put_row128(A, r, pk);
          fence_proxy_async_smem();
        } else {  // dS row -> this thread's TMEM lane, the A operand of dQ += dS K_j
          const uint32_t dcol = tmem + lane_off + BW_G + t * 128 + BW_DS;
          tmem_st32(dcol, pk);
          tmem_st32(dcol + 32, pk + 32);
          tmem_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->ds_ready[t]);
        if (DKDV) {
          my_lse = nl;
          my_delta = nd;
        }
      }
      // ---- results
      if (ok && mbar_wait(&bars->done, 0, abort_flag)) {
        tc_fence_after();
        const int row = (2 * pair + t) * 128 + r;  // dkdv: key; dq: query
        const bool st = row < T;
        const long ld = 3L * C;
        bf16* rowp = dqkv + ((long)row_base + (st ? row : 0)) * ld;
        const uint32_t g = tmem + lane_off + BW_G + t * 128;
        if (DKDV) {
          store_row64(g, rowp + C + h * D, scale, st);            // dK
          store_row64(g + 64, rowp + 2 * C + h * D, 1.f, st);     // dV
        } else {
          store_row64(g, rowp + h * D, scale, st);                // dQ
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
// dQ = scale * dS K from the dS tiles the dK/dV kernel stored (head dim 64).
// CTA = (query tile i, batch*head); key tiles j <= i stream through a ring of
// DQ_STAGES stages, each holding the dS tile (two 64-key atoms: the K-major A
// operand, M = queries) and K_j (the MN-major B operand).  Warp 0 issues the TMA
// loads, one thread of warp 1 the MMAs into a 64-column TMEM accumulator; warps
// 2..5 read it back (one query row each), scale and store bf16.  The key tiles are
// summed in increasing order, so the result does not depend on scheduling.
// Reference math: dtrain/autograd.py:239-247 (gq = gs k).
// =============================================================================
constexpr int DQ_THREADS = 192;
constexpr int DQ_STAGES = 4;
constexpr int DQ_STAGE_BYTES = PBYTES + TILE;  // 32 KB dS + 16 KB K
constexpr int DQ_OFF_BAR = DQ_STAGES * DQ_STAGE_BYTES;
constexpr int DQ_SMEM = DQ_OFF_BAR + 256 + 1024;

struct DqBars {
  uint64_t full[DQ_STAGES], empty[DQ_STAGES];
  uint64_t done;
  uint32_t tmem_slot;
  int abort_flag;
};

__global__ void __launch_bounds__(DQ_THREADS, 1)
    dq_from_ds_kernel(const __grid_constant__ CUtensorMap tmDS, const __grid_constant__ CUtensorMap tmQKV,
                      bf16* __restrict__ dqkv, int T, int H, float scale) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  DqBars* bars = reinterpret_cast<DqBars*>(smem + DQ_OFF_BAR);
  volatile int* abort_flag = &bars->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = (T + 127) / 128;
  const int i = nt - 1 - (int)blockIdx.x;  // the longest query tiles first
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int C = H * D;
  const int nj = i + 1;  // causal: key tiles 0..i

  if (threadIdx.x == 0) {
    for (int k = 0; k < DQ_STAGES; ++k) {
      mbar_init(&bars->full[k], 1);
      mbar_init(&bars->empty[k], 1);
    }
    mbar_init(&bars->done, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmDS);
    tma_prefetch_desc(&tmQKV);
  }
  if (warp == 1) tmem_alloc(&bars->tmem_slot, 64);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int j = 0; j < nj; ++j) {
        const int st = j % DQ_STAGES;
        const uint32_t ph = ((j / DQ_STAGES) & 1) ^ 1;
        if (!mbar_wait(&bars->empty[st], ph, abort_flag)) break;
        uint8_t* stage = smem + st * DQ_STAGE_BYTES;
        mbar_arrive_expect_tx(&bars->full[st], DQ_STAGE_BYTES);
        tma_load_3d(&tmDS, stage, &bars->full[st], j * 128, i * 128, bh);
        tma_load_3d(&tmDS, stage + 16384, &bars->full[st], j * 128 + 64, i * 128, bh);
        tma_load_2d(&tmQKV, stage + PBYTES, &bars->full[st], C + h * D, b * T + j * 128);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(128, D, false, true);  // A K-major (dS), B MN-major (K)
      bool ok = true;
      for (int j = 0; j < nj && ok; ++j) {
        const int st = j % DQ_STAGES;
        if (!mbar_wait(&bars->full[st], (j / DQ_STAGES) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a = smem_u32(smem + st * DQ_STAGE_BYTES), kb = a + PBYTES;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_f16(tmem, make_sw128_desc(a + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                     make_sw128_desc(kb + kk * 2048, 8192, 1024), idesc, (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&bars->empty[st]);
      }
      if (ok) tc_commit(&bars->done);
    }
  } else {
    const int q = warp & 3;  // TMEM lanes 32q .. 32q+31 belong to warps with warp % 4 == q
    const int row = i * 128 + q * 32 + lane;
    if (mbar_wait(&bars->done, 0, abort_flag)) {
      tc_fence_after();
      bf16* dst = dqkv + ((long)b * T + (row < T ? row : 0)) * 3L * C + h * D;
      store_row64(tmem + ((uint32_t)(q * 32) << 16), dst, scale, row < T);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
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

void attn_delta64(torch::Tensor out, torch::Tensor dout, torch::Tensor delta, int64_t B, int64_t T, int64_t H);

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

// dS scratch [B*H][T][Tp] bf16 (Tp = T rounded up to 128 keys) as a 3-D tensor map
// with 64-key x 128-query boxes: rows past T and keys past T clip (stores) or read
// as zero (loads), and one (b, h) never spills into the next.
static CUtensorMap ds_map(const torch::Tensor& ds, long BH, long T, long Tp) {
  CUtensorMap m;
  cuuint64_t dims[3] = {(cuuint64_t)Tp, (cuuint64_t)T, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)Tp * 2, (cuuint64_t)T * Tp * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn_attn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, ds.data_ptr(), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "attention: dS tensor map encode failed ", (int)r);
  return m;
}

// tcgen05 backward for head dim 64, into dqkv [B*T, 3*H*64]:
//   delta = rowsum(dO * O)                                   (delta_kernel)
//   dK, dV, and every causal dS tile stored to a scratch      (bwd_tc_kernel<true>)
//   dQ = scale * dS K                                          (dq_from_ds_kernel)
// DTB_ATTN_DQ=recompute selects the older dQ kernel that recomputes P and dP
// (bwd_tc_kernel<false>, which also writes delta) ahead of dK/dV instead.
void attn_bwd_tc(torch::Tensor qkv, torch::Tensor out, torch::Tensor dout, torch::Tensor lse, torch::Tensor delta,
                 torch::Tensor dqkv, int64_t B, int64_t T, int64_t H) {
  using namespace attn_tc;
  TORCH_CHECK(dout.is_contiguous() && dout.numel() == B * T * H * D, "attn_bwd_tc: dout must be [B*T, H*64]");
  TORCH_CHECK(out.is_contiguous() && out.numel() == B * T * H * D && out.scalar_type() == at::kBFloat16,
              "attn_bwd_tc: out must be bf16 [B*T, H*64]");
  TORCH_CHECK(delta.is_contiguous() && delta.numel() == B * H * T && delta.scalar_type() == at::kFloat,
              "attn_bwd_tc: delta must be fp32 [B*H, T]");
  c10::cuda::CUDAGuard guard(qkv.device());
  bind_device_context(qkv.get_device());
  CUtensorMap mq = attn_map(qkv, B * T, 3 * H * D);
  CUtensorMap md = attn_map(dout, B * T, H * D);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(bwd_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, BW_SMEM);
    cudaFuncSetAttribute(bwd_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, BW_SMEM);
    cudaFuncSetAttribute(dq_from_ds_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DQ_SMEM);
    attr = true;
  }
  static const bool recompute = [] {
    const char* e = std::getenv("DTB_ATTN_DQ");
    return e && std::string(e) == "recompute";
  }();
  const int nt = (int)((T + 127) / 128);
  dim3 grid((unsigned)((nt + 1) / 2), (unsigned)(B * H));
  const float scale = 0.125f;                               // 1/sqrt(64)
  const float sl2 = (float)(1.4426950408889634 / 8.0);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto* dq = reinterpret_cast<bf16*>(dqkv.data_ptr());
  auto* o = reinterpret_cast<const bf16*>(out.data_ptr());
  auto* g = reinterpret_cast<const bf16*>(dout.data_ptr());
  if (recompute) {
    bwd_tc_kernel<false><<<grid, BW_THREADS, BW_SMEM, st>>>(mq, md, md, lse.data_ptr<float>(),
                                                            delta.data_ptr<float>(), o, g, dq, (int)T, (int)H, sl2,
                                                            scale, 0);
    bwd_tc_kernel<true><<<grid, BW_THREADS, BW_SMEM, st>>>(mq, md, md, lse.data_ptr<float>(),
                                                           delta.data_ptr<float>(), o, g, dq, (int)T, (int)H, sl2,
                                                           scale, 0);
    count_launch(2);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  const long Tp = (long)nt * 128;
  auto ds = torch::empty({B * H, T, Tp}, qkv.options());
  CUtensorMap mds = ds_map(ds, B * H, T, Tp);
  attn_delta64(out, dout, delta, B, T, H);
  bwd_tc_kernel<true><<<grid, BW_THREADS, BW_SMEM, st>>>(mq, md, mds, lse.data_ptr<float>(), delta.data_ptr<float>(),
                                                         o, g, dq, (int)T, (int)H, sl2, scale, 1);
  dq_from_ds_kernel<<<dim3((unsigned)nt, (unsigned)(B * H)), DQ_THREADS, DQ_SMEM, st>>>(mds, mq, dq, (int)T, (int)H,
                                                                                        scale);
  count_launch(2);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

DTB_DEFINE_STATUS_READER(status_attention_tc)

}  // namespace dtb
