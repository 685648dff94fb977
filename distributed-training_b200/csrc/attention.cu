// Causal self-attention, flash-style, reading q/k/v straight from the qkv GEMM output.
//
// Replaces dtrain/autograd.py:226-247 (causal_attention), which materialises the
// B*H*T*T score matrix, and the split/transposes around it (dtrain/nn.py:98-117).
// Layout: qkv is [B*T, 3*H*D] bf16 as produced by the qkv Linear ([B,T,3,H,D]);
// the output is [B*T, H*D] bf16 and is consumed by the proj Linear as is.
//
// Forward: one CTA per (64-query tile, batch*head), 4 warps x 16 query rows;
// K/V tiles of 64 keys are double-buffered in XOR-swizzled shared memory with
// cp.async; online softmax in the log2 domain (exp2f with log2(e)/sqrt(D) folded
// into one scale); causal tiles above the diagonal are skipped.  The per-row
// log-sum-exp (log2 domain) is saved for the backward.
//
// Backward is deterministic (no atomics): one kernel owns a key tile and
// accumulates dK, dV over the query tiles that see it; a second kernel owns a
// query tile and accumulates dQ over its key tiles.  Both recompute P from the
// saved log-sum-exp.  delta = rowsum(dO * O) is computed once by a small kernel (the head-dim-64
// tcgen05 path computes it inside its dQ kernel instead).
//
// Tensor-core path: warp-level mma.sync m16n8k16 (bf16 in, fp32 accumulate).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace dtb {

namespace attn {

constexpr int BQ = 64;
constexpr int BKV = 64;
constexpr int kThreads = 128;

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Byte offset of element (row, col) in a [rows][D] bf16 tile with 16-byte chunks
// XOR-swizzled by (row & 7) so that ldmatrix row reads hit distinct banks.
template <int D>
__device__ __forceinline__ uint32_t swz(int row, int col) {
  const int chunk = col >> 3;
  const int sw = (chunk & ~7) | ((chunk ^ row) & 7);
  return (uint32_t)(row * (D * 2) + sw * 16 + (col & 7) * 2);
}

// Copy rows [r0, r0+64) of a [T, ld] matrix (columns [0, D)) into a swizzled tile; rows >= T are zero.
template <int D>
__device__ __forceinline__ void load_tile(uint32_t sbase, const bf16* g, long ld, int r0, int T) {
  constexpr int CH = D / 8;  // 16-byte chunks per row
#pragma unroll
  for (int k = 0; k < (64 * CH) / kThreads; ++k) {
    const int idx = threadIdx.x + k * kThreads;
    const int r = idx / CH, c = (idx % CH) * 8;
    const bool ok = (r0 + r) < T;
    const bf16* src = g + (long)(ok ? (r0 + r) : 0) * ld + c;
    cp_async16(sbase + swz<D>(r, c), src, ok);
  }
}

__device__ __forceinline__ uint32_t pack2(float a, float b) { return pack_bf16x2(a, b); }

__device__ __forceinline__ float quad_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
  return v;
}
__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  return v;
}

// Load the A fragments of a 16 x D strip (rows r0..r0+15 of a swizzled tile).
template <int D>
__device__ __forceinline__ void load_a_frags(uint32_t (&f)[D / 16][4], uint32_t sbase, int r0, int lane) {
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) ldsm_x4(f[kk], sbase + swz<D>(r0 + (lane & 15), kk * 16 + (lane >> 4) * 8));
}

// acc[8][4] (16 rows x 64 cols) = A(16 x D, fragments) * B^T where B is a 64 x D swizzled tile (rows = output cols).
template <int D>
__device__ __forceinline__ void mma_abt(float (&acc)[8][4], const uint32_t (&af)[D / 16][4], uint32_t sB, int lane) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t r[4];
      const int row = np * 16 + (lane & 7) + ((lane >> 4) << 3);
      const int col = kk * 16 + ((lane >> 3) & 1) * 8;
      ldsm_x4(r, sB + swz<D>(row, col));
      mma16816(acc[2 * np], af[kk], r[0], r[1]);
      mma16816(acc[2 * np + 1], af[kk], r[2], r[3]);
    }
  }
}

// out[D/8][4] (16 rows x D) += P(16 x 64, packed A fragments) * B where B is a 64 x D swizzled tile (rows = k).
template <int D>
__device__ __forceinline__ void mma_pb(float (&out)[D / 8][4], const uint32_t (&pf)[4][4], uint32_t sB, int lane) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
    for (int dp = 0; dp < D / 16; ++dp) {
      uint32_t r[4];
      const int row = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
      const int col = dp * 16 + (lane >> 4) * 8;
      ldsm_x4_t(r, sB + swz<D>(row, col));
      mma16816(out[2 * dp], pf[kk], r[0], r[1]);
      mma16816(out[2 * dp + 1], pf[kk], r[2], r[3]);
    }
  }
}

// Convert a 16 x 64 fp32 accumulator into bf16 A fragments (k = the 64 columns).
__device__ __forceinline__ void acc_to_afrag(uint32_t (&pf)[4][4], const float (&s)[8][4]) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    pf[kk][0] = pack2(s[2 * kk][0], s[2 * kk][1]);
    pf[kk][1] = pack2(s[2 * kk][2], s[2 * kk][3]);
    pf[kk][2] = pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
    pf[kk][3] = pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
  }
}

template <int D>
__global__ void __launch_bounds__(kThreads)
    fwd_kernel(const bf16* __restrict__ qkv, bf16* __restrict__ out, float* __restrict__ lse2, int T, int H,
               float sl2) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int TILE = 64 * D * 2;
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + TILE, sV0 = sQ + 3 * TILE;  // K: [2] tiles, V: [2] tiles
  const int qt = gridDim.x - 1 - blockIdx.x;             // heavy (late) query tiles first
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long ld = 3L * H * D;
  const bf16* qb = qkv + (long)b * T * ld + (long)h * D;
  const bf16* kb = qb + (long)H * D;
  const bf16* vb = qb + 2L * H * D;
  const int q0 = qt * BQ;

  load_tile<D>(sQ, qb, ld, q0, T);
  load_tile<D>(sK0, kb, ld, 0, T);
  load_tile<D>(sV0, vb, ld, 0, T);
  cp_commit();

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  uint32_t qf[D / 16][4];
  const int g = lane >> 2, cq = (lane & 3) * 2;
  const int qrow0 = q0 + warp * 16 + g;  // this thread's rows: qrow0, qrow0 + 8

  const int nkv = qt + 1;
  for (int j = 0; j < nkv; ++j) {
    if (j + 1 < nkv) {
      const int nb = (j + 1) & 1;
      load_tile<D>(sK0 + nb * TILE, kb, ld, (j + 1) * BKV, T);
      load_tile<D>(sV0 + nb * TILE, vb, ld, (j + 1) * BKV, T);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (j == 0) load_a_frags<D>(qf, sQ, warp * 16, lane);
    const uint32_t sK = sK0 + (j & 1) * TILE, sV = sV0 + (j & 1) * TILE;
    float s[8][4];
    mma_abt<D>(s, qf, sK, lane);
    // scale, mask, running max
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = j * BKV + n * 8 + cq + (e & 1);
        const int qr = qrow0 + (e >> 1) * 8;
        float x = s[n][e] * sl2;
        if (key > qr || key >= T) x = -INFINITY;
        s[n][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = quad_max(mx[r]);
      const float mn = fmaxf(mrow[r], mx[r]);
      alpha[r] = (mrow[r] == -INFINITY) ? 0.f : exp2f(mrow[r] - mn);
      mrow[r] = mn;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float base = mrow[e >> 1];
        const float p = (base == -INFINITY) ? 0.f : exp2f(s[n][e] - base);
        s[n][e] = p;
        rs[e >> 1] += p;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) lrow[r] = lrow[r] * alpha[r] + rs[r];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
    uint32_t pf[4][4];
    acc_to_afrag(pf, s);
    mma_pb<D>(o, pf, sV, lane);
    __syncthreads();
  }
  // finalize
#pragma unroll
  for (int r = 0; r < 2; ++r) lrow[r] = quad_sum(lrow[r]);
  const long ldo = (long)H * D;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qr = qrow0 + r * 8;
    if (qr >= T) continue;
    const float inv = lrow[r] > 0.f ? 1.f / lrow[r] : 0.f;
    bf16* orow = out + ((long)b * T + qr) * ldo + (long)h * D;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      *reinterpret_cast<uint32_t*>(orow + i * 8 + cq) = pack2(o[i][2 * r] * inv, o[i][2 * r + 1] * inv);
    }
    if ((lane & 3) == 0) lse2[(long)bh * T + qr] = mrow[r] + log2f(lrow[r]);
  }
}

// delta[bh, t] = sum_d dO[t, h, d] * O[t, h, d]
// D/8 consecutive lanes share a row: each loads 16 bytes of O and of dO (8 values),
// sums its 8 products in order, and the lanes then combine with a fixed shuffle tree.
// Rows are numbered (b, h, t) with t fastest, so the delta writes of a warp are
// contiguous; every thread walks two rows per iteration (four 16-byte loads in flight)
// over a grid-stride loop.
template <int D>
__global__ void __launch_bounds__(256)
    delta_kernel(const bf16* __restrict__ o, const bf16* __restrict__ dout, float* __restrict__ delta, int B, int T,
                 int H) {
  constexpr int L = D / 8;  // lanes per row
  const int sub = threadIdx.x % L;
  const long nrows = (long)B * H * T;
  const long groups = (long)gridDim.x * (blockDim.x / L);
  const long stride = (long)H * D;  // elements between consecutive t of one (b, h)
  auto row_ptr = [&](long r, const bf16* base) {
    const long t = r % T, bh = r / T;
    const long b = bh / H, h = bh % H;
    return base + (b * T + t) * stride + h * D + sub * 8;
  };
  auto dot8 = [](const uint4& a, const uint4& g) {
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, gw[4] = {g.x, g.y, g.z, g.w};
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      acc = fmaf(__uint_as_float(aw[e] << 16), __uint_as_float(gw[e] << 16), acc);
      acc = fmaf(__uint_as_float(aw[e] & 0xffff0000u), __uint_as_float(gw[e] & 0xffff0000u), acc);
    }
    return acc;
  };
  const long first = (long)blockIdx.x * (blockDim.x / L) + threadIdx.x / L;  // this lane's row group
  const long in_warp = (threadIdx.x / L) % (32 / L);                         // its index inside the warp
  // the loop runs on the warp's first row group, so every lane of a warp takes the same
  // number of iterations and the shuffles below always see the whole warp
  for (long w0 = first - in_warp; w0 < nrows; w0 += 2 * groups) {
    const long r = w0 + in_warp, r2 = r + groups;
    const bool ok = r < nrows, ok2 = r2 < nrows;
    uint4 a{}, g{}, a2{}, g2{};
    if (ok) {
      a = *reinterpret_cast<const uint4*>(row_ptr(r, o));
      g = *reinterpret_cast<const uint4*>(row_ptr(r, dout));
    }
    if (ok2) {
      a2 = *reinterpret_cast<const uint4*>(row_ptr(r2, o));
      g2 = *reinterpret_cast<const uint4*>(row_ptr(r2, dout));
    }
    float s = dot8(a, g), s2 = dot8(a2, g2);
#pragma unroll
    for (int k = L / 2; k > 0; k >>= 1) {
      s += __shfl_xor_sync(0xffffffffu, s, k);
      s2 += __shfl_xor_sync(0xffffffffu, s2, k);
    }
    if (sub == 0) {
      if (ok) delta[r] = s;
      if (ok2) delta[r2] = s2;
    }
  }
}

// Grid of the delta kernel: enough 256-thread blocks for every SM to keep a few resident.
inline unsigned delta_grid(long nrows, int D) {
  const long rows_per_block = 256 / (D / 8);
  return (unsigned)std::max<long>(1, std::min<long>((nrows + 2 * rows_per_block - 1) / (2 * rows_per_block), 148 * 8));
}

// dK, dV for one 64-key tile; warps own 16 keys each.
template <int D>
__global__ void __launch_bounds__(kThreads)
    bwd_dkdv_kernel(const bf16* __restrict__ qkv, const bf16* __restrict__ dout, const float* __restrict__ lse2,
                    const float* __restrict__ delta, bf16* __restrict__ dqkv, int T, int H, float sl2, float scale) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int TILE = 64 * D * 2;
  const uint32_t sK = smem_u32(smem), sV = sK + TILE;
  const uint32_t sQ0 = sK + 2 * TILE, sO0 = sK + 4 * TILE;  // Q: [2], dO: [2]
  float* sL = reinterpret_cast<float*>(smem + 6 * TILE);     // [2][64] lse2
  float* sD = sL + 128;                                       // [2][64] delta
  const int kt = blockIdx.x;
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long ld = 3L * H * D, ldo = (long)H * D;
  const bf16* qb = qkv + (long)b * T * ld + (long)h * D;
  const bf16* kb = qb + (long)H * D;
  const bf16* vb = qb + 2L * H * D;
  const bf16* ob = dout + (long)b * T * ldo + (long)h * D;
  const float* lb = lse2 + (long)bh * T;
  const float* db = delta + (long)bh * T;
  const int k0 = kt * BKV;
  const int nqt = (T + BQ - 1) / BQ;

  auto load_q = [&](int i, int buf) {
    load_tile<D>(sQ0 + buf * TILE, qb, ld, i * BQ, T);
    load_tile<D>(sO0 + buf * TILE, ob, ldo, i * BQ, T);
    if (threadIdx.x < 64) {
      const int t = i * BQ + threadIdx.x;
      sL[buf * 64 + threadIdx.x] = t < T ? lb[t] : 0.f;
      sD[buf * 64 + threadIdx.x] = t < T ? db[t] : 0.f;
    }
  };
  load_tile<D>(sK, kb, ld, k0, T);
  load_tile<D>(sV, vb, ld, k0, T);
  load_q(kt, 0);
  cp_commit();

  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;
  uint32_t kf[D / 16][4], vf[D / 16][4];
  const int g = lane >> 2, cq = (lane & 3) * 2;
  const int krow0 = k0 + warp * 16 + g;

  for (int i = kt; i < nqt; ++i) {
    const int buf = (i - kt) & 1;
    if (i + 1 < nqt) {
      __syncthreads();  // the other buffer's previous contents are consumed
      load_q(i + 1, buf ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (i == kt) {
      load_a_frags<D>(kf, sK, warp * 16, lane);
      load_a_frags<D>(vf, sV, warp * 16, lane);
    }
    const uint32_t sQ = sQ0 + buf * TILE, sO = sO0 + buf * TILE;
    const float* L = sL + buf * 64;
    const float* Dl = sD + buf * 64;
    // P^T (16 keys x 64 queries)
    float pt[8][4];
    mma_abt<D>(pt, kf, sQ, lane);
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qc = n * 8 + cq + (e & 1);
        const int q = i * BQ + qc;
        const int key = krow0 + (e >> 1) * 8;
        pt[n][e] = (q < key || q >= T) ? 0.f : exp2f(pt[n][e] * sl2 - L[qc]);
      }
    }
    // dP^T = V dO^T
    float dpt[8][4];
    mma_abt<D>(dpt, vf, sO, lane);
    // dV += P^T dO
    uint32_t pf[4][4];
    acc_to_afrag(pf, pt);
    mma_pb<D>(dv, pf, sO, lane);
    // dS^T = P^T * (dP^T - delta)
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) dpt[n][e] = pt[n][e] * (dpt[n][e] - Dl[n * 8 + cq + (e & 1)]);
    acc_to_afrag(pf, dpt);
    mma_pb<D>(dk, pf, sQ, lane);
  }
  // write dK (scaled) and dV
  bf16* dkb = dqkv + (long)b * T * ld + (long)H * D + (long)h * D;
  bf16* dvb = dkb + (long)H * D;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int kr = krow0 + r * 8;
    if (kr >= T) continue;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      *reinterpret_cast<uint32_t*>(dkb + (long)kr * ld + i * 8 + cq) =
          pack2(dk[i][2 * r] * scale, dk[i][2 * r + 1] * scale);
      *reinterpret_cast<uint32_t*>(dvb + (long)kr * ld + i * 8 + cq) = pack2(dv[i][2 * r], dv[i][2 * r + 1]);
    }
  }
}

// dQ for one 64-query tile; warps own 16 queries each.
template <int D>
__global__ void __launch_bounds__(kThreads)
    bwd_dq_kernel(const bf16* __restrict__ qkv, const bf16* __restrict__ dout, const float* __restrict__ lse2,
                  const float* __restrict__ delta, bf16* __restrict__ dqkv, int T, int H, float sl2, float scale) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int TILE = 64 * D * 2;
  const uint32_t sQ = smem_u32(smem), sO = sQ + TILE;
  const uint32_t sK0 = sQ + 2 * TILE, sV0 = sQ + 4 * TILE;
  const int qt = gridDim.x - 1 - blockIdx.x;
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long ld = 3L * H * D, ldo = (long)H * D;
  const bf16* qb = qkv + (long)b * T * ld + (long)h * D;
  const bf16* kb = qb + (long)H * D;
  const bf16* vb = qb + 2L * H * D;
  const bf16* ob = dout + (long)b * T * ldo + (long)h * D;
  const int q0 = qt * BQ;
  const int g = lane >> 2, cq = (lane & 3) * 2;
  const int qrow0 = q0 + warp * 16 + g;

  load_tile<D>(sQ, qb, ld, q0, T);
  load_tile<D>(sO, ob, ldo, q0, T);
  load_tile<D>(sK0, kb, ld, 0, T);
  load_tile<D>(sV0, vb, ld, 0, T);
  cp_commit();
  float L[2], Dl[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int q = qrow0 + r * 8;
    L[r] = q < T ? lse2[(long)bh * T + q] : 0.f;
    Dl[r] = q < T ? delta[(long)bh * T + q] : 0.f;
  }
  float dq[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dq[i][e] = 0.f;
  uint32_t qf[D / 16][4], of[D / 16][4];

  const int nkv = qt + 1;
  for (int j = 0; j < nkv; ++j) {
    if (j + 1 < nkv) {
      const int nb = (j + 1) & 1;
      load_tile<D>(sK0 + nb * TILE, kb, ld, (j + 1) * BKV, T);
      load_tile<D>(sV0 + nb * TILE, vb, ld, (j + 1) * BKV, T);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
      load_a_frags<D>(qf, sQ, warp * 16, lane);
      load_a_frags<D>(of, sO, warp * 16, lane);
    }
    const uint32_t sK = sK0 + (j & 1) * TILE, sV = sV0 + (j & 1) * TILE;
    float p[8][4];
    mma_abt<D>(p, qf, sK, lane);
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = j * BKV + n * 8 + cq + (e & 1);
        const int qr = qrow0 + (e >> 1) * 8;
        p[n][e] = (key > qr || key >= T || qr >= T) ? 0.f : exp2f(p[n][e] * sl2 - L[e >> 1]);
      }
    float dp[8][4];
    mma_abt<D>(dp, of, sV, lane);
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) dp[n][e] = p[n][e] * (dp[n][e] - Dl[e >> 1]);
    uint32_t pf[4][4];
    acc_to_afrag(pf, dp);
    mma_pb<D>(dq, pf, sK, lane);
    __syncthreads();
  }
  bf16* dqb = dqkv + (long)b * T * ld + (long)h * D;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qr = qrow0 + r * 8;
    if (qr >= T) continue;
#pragma unroll
    for (int i = 0; i < D / 8; ++i)
      *reinterpret_cast<uint32_t*>(dqb + (long)qr * ld + i * 8 + cq) =
          pack2(dq[i][2 * r] * scale, dq[i][2 * r + 1] * scale);
  }
}

}  // namespace attn

// ------------------------------------------------------------------ host
static void check_qkv(const torch::Tensor& qkv, int64_t B, int64_t T, int64_t H, int64_t D) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.is_contiguous(), "attention: qkv bf16");
  TORCH_CHECK(qkv.numel() == B * T * 3 * H * D, "attention: qkv must be [B*T, 3*H*D]");
  TORCH_CHECK(D == 64 || D == 128, "attention: head dim must be 64 or 128");
}

void attn_fwd_tc(torch::Tensor qkv, torch::Tensor out, torch::Tensor lse, int64_t B, int64_t T, int64_t H);

// Returns (out [B*T, H*D] bf16, lse2 [B*H, T] fp32).  Head dim 64 runs the tcgen05
// kernel (attention_tc.cu) unless `legacy` asks for the mma.sync kernel below.
std::vector<torch::Tensor> attn_fwd(torch::Tensor qkv, int64_t B, int64_t T, int64_t H, int64_t D, bool legacy) {
  check_qkv(qkv, B, T, H, D);
  c10::cuda::CUDAGuard guard(qkv.device());
  auto out = torch::empty({B * T, H * D}, qkv.options());
  auto lse = torch::empty({B * H, T}, qkv.options().dtype(at::kFloat));
  if (D == 64 && !legacy) {
    attn_fwd_tc(qkv, out, lse, B, T, H);
    return {out, lse};
  }
  const float sl2 = (float)(1.0 / std::sqrt((double)D) * 1.4426950408889634);
  dim3 grid((unsigned)((T + attn::BQ - 1) / attn::BQ), (unsigned)(B * H));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto* q = reinterpret_cast<const bf16*>(qkv.data_ptr());
  auto* o = reinterpret_cast<bf16*>(out.data_ptr());
  if (D == 64) {
    const int smem = 5 * 64 * 64 * 2;
    attn::fwd_kernel<64><<<grid, attn::kThreads, smem, st>>>(q, o, lse.data_ptr<float>(), (int)T, (int)H, sl2);
  } else {
    const int smem = 5 * 64 * 128 * 2;
    auto k = attn::fwd_kernel<128>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    k<<<grid, attn::kThreads, smem, st>>>(q, o, lse.data_ptr<float>(), (int)T, (int)H, sl2);
  }
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {out, lse};
}

// delta = rowsum(dout * out) [B*H, T] for head dim 64 (one warp per row).
void attn_delta64(torch::Tensor out, torch::Tensor dout, torch::Tensor delta, int64_t B, int64_t T, int64_t H) {
  const long warps = B * T * H;
  attn::delta_kernel<64><<<attn::delta_grid(warps, 64), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(out.data_ptr()), reinterpret_cast<const bf16*>(dout.data_ptr()),
      delta.data_ptr<float>(), (int)B, (int)T, (int)H);
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Returns dqkv [B*T, 3*H*D] bf16.
void attn_bwd_tc(torch::Tensor qkv, torch::Tensor out, torch::Tensor dout, torch::Tensor lse, torch::Tensor delta,
                 torch::Tensor dqkv, int64_t B, int64_t T, int64_t H);

// Head dim 64 runs the tcgen05 backward kernels (attention_tc.cu) unless `legacy`.
torch::Tensor attn_bwd(torch::Tensor qkv, torch::Tensor out, torch::Tensor dout, torch::Tensor lse, int64_t B,
                       int64_t T, int64_t H, int64_t D, bool legacy) {
  check_qkv(qkv, B, T, H, D);
  if (D == 64 && !legacy) {
    TORCH_CHECK(dout.is_contiguous() && dout.scalar_type() == at::kBFloat16 && dout.numel() == B * T * H * D,
                "attention: dout");
    c10::cuda::CUDAGuard guard(qkv.device());
    auto dqkv = torch::empty_like(qkv);
    auto delta = torch::empty({B * H, T}, qkv.options().dtype(at::kFloat));
    attn_bwd_tc(qkv, out.contiguous(), dout, lse, delta, dqkv, B, T, H);
    return dqkv;
  }
  TORCH_CHECK(dout.is_contiguous() && dout.scalar_type() == at::kBFloat16 && dout.numel() == B * T * H * D,
              "attention: dout");
  c10::cuda::CUDAGuard guard(qkv.device());
  auto dqkv = torch::empty_like(qkv);
  auto delta = torch::empty({B * H, T}, qkv.options().dtype(at::kFloat));
  const float scale = (float)(1.0 / std::sqrt((double)D));
  const float sl2 = scale * 1.4426950408889634f;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto* q = reinterpret_cast<const bf16*>(qkv.data_ptr());
  auto* o = reinterpret_cast<const bf16*>(out.data_ptr());
  auto* g = reinterpret_cast<const bf16*>(dout.data_ptr());
  auto* dq = reinterpret_cast<bf16*>(dqkv.data_ptr());
  const long warps = B * T * H;
  dim3 grid((unsigned)((T + 63) / 64), (unsigned)(B * H));
  if (D == 64) {
    attn::delta_kernel<64><<<attn::delta_grid(warps, 64), 256, 0, st>>>(o, g, delta.data_ptr<float>(),
                                                                                 (int)B, (int)T, (int)H);
    const int smem_kv = 6 * 64 * 64 * 2 + 4 * 64 * 4;
    const int smem_q = 6 * 64 * 64 * 2;
    auto k1 = attn::bwd_dkdv_kernel<64>;
    auto k2 = attn::bwd_dq_kernel<64>;
    cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_kv);
    cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_q);
    k1<<<grid, attn::kThreads, smem_kv, st>>>(q, g, lse.data_ptr<float>(), delta.data_ptr<float>(), dq, (int)T,
                                              (int)H, sl2, scale);
    k2<<<grid, attn::kThreads, smem_q, st>>>(q, g, lse.data_ptr<float>(), delta.data_ptr<float>(), dq, (int)T,
                                             (int)H, sl2, scale);
  } else {
    attn::delta_kernel<128><<<attn::delta_grid(warps, 128), 256, 0, st>>>(o, g, delta.data_ptr<float>(),
                                                                                  (int)B, (int)T, (int)H);
    const int smem_kv = 6 * 64 * 128 * 2 + 4 * 64 * 4;
    const int smem_q = 6 * 64 * 128 * 2;
    auto k1 = attn::bwd_dkdv_kernel<128>;
    auto k2 = attn::bwd_dq_kernel<128>;
    cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_kv);
    cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_q);
    k1<<<grid, attn::kThreads, smem_kv, st>>>(q, g, lse.data_ptr<float>(), delta.data_ptr<float>(), dq, (int)T,
                                              (int)H, sl2, scale);
    k2<<<grid, attn::kThreads, smem_q, st>>>(q, g, lse.data_ptr<float>(), delta.data_ptr<float>(), dq, (int)T,
                                             (int)H, sl2, scale);
  }
  count_launch(3);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dqkv;
}

DTB_DEFINE_STATUS_READER(status_attention)

}  // namespace dtb
