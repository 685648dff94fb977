// LayerNorm forward/backward and the deterministic column-sum used for bias grads.
//
// Mirrors dtrain/autograd.py:207-223 (layer_norm): population variance of the
// centred input, rstd = 1/sqrt(var + eps), y = xhat*w + b; backward
//   dx = rstd * (g*w - mean(g*w) - xhat * mean(g*w*xhat))
// plus row sums for dw and db.  Here x/y/dy/dx are bf16 [rows, C], statistics and
// parameter gradients are fp32.  The backward also adds the residual-stream
// gradient (dresid) so the residual add costs no extra pass.
//
// Determinism: dw/db are reduced in two fixed-order stages (per-block partials in
// a workspace, then a column-wise sum over blocks in block order), never with
// float atomics, so repeated runs give identical bits.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "dtb_noalloc.h"

namespace dtb {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void ld8(const bf16* p, float* v) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ void st8(bf16* p, const float* v) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ void unpack8(const uint4& u, float* v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// Two rows per warp (both rows' loads in flight together); lane l owns 8-element
// chunks l, l+32, l+64, ... (NCH chunks) of each row.
template <int NCH>
__global__ void ln_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w, const bf16* __restrict__ b,
                              bf16* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out,
                              int rows, int C, float eps) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int r0 = warp * 2;
  if (r0 >= rows) return;
  uint4 raw[2][NCH];
#pragma unroll
  for (int k = 0; k < 2; ++k)
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < C && r0 + k < rows) raw[k][c] = *reinterpret_cast<const uint4*>(x + (long)(r0 + k) * C + col);
    }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int r = r0 + k;
    if (r >= rows) break;
    float v[NCH][8];
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < C) {
        unpack8(raw[k][c], v[c]);
#pragma unroll
        for (int j = 0; j < 8; ++j) s += v[c][j];
      }
    }
    const float mu = warp_sum(s) / C;
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < C) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float d = v[c][j] - mu;
          ss += d * d;
        }
      }
    }
    const float var = warp_sum(ss) / C;
    const float rs = rsqrtf(var + eps);
    bf16* yr = y + (long)r * C;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < C) {
        float wv[8], bv[8], o[8];
        ld8(w + col, wv);
        ld8(b + col, bv);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = (v[c][j] - mu) * rs * wv[j] + bv[j];
        st8(yr + col, o);
      }
    }
    if (lane == 0) {
      mean_out[r] = mu;
      rstd_out[r] = rs;
    }
  }
}

constexpr int kLnBwdWarps = 8;
constexpr int kLnBwdRowsPerBlock = 64;

// Dynamic shared memory of ln_bwd_kernel<NCH>: per-warp column accumulators
// [3][NCH * 256] (rows padded to whole 256-column chunks).
static inline size_t ln_bwd_smem(int nch) { return (size_t)kLnBwdWarps * 3 * nch * 256 * sizeof(float); }

// Block b handles rows [b*64, b*64+64); warp k handles rows b*64 + k, +8, ... and
// prefetches its next row while it computes the current one (the row's dy, x and
// dresid stay in registers between the two passes, nothing is re-read).  Column
// sums of g*xhat (dw), g (db) and - when part_r is given - of the residual
// gradient dresid (the bias gradient of the layer that produced it) accumulate in
// per-warp shared-memory rows, then combine in warp order into per-block partials
// [gridDim.x, C].
template <int NCH>
__global__ void __launch_bounds__(kLnBwdWarps * 32, 2)
    ln_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x, const bf16* __restrict__ w,
                  const float* __restrict__ mean, const float* __restrict__ rstd, const bf16* __restrict__ dresid,
                  bf16* __restrict__ dx, float* __restrict__ part_w, float* __restrict__ part_b,
                  float* __restrict__ part_r, int rows, int C) {
  constexpr int RS = NCH * 256;  // accumulator row stride (floats)
  extern __shared__ float sm[];  // [kLnBwdWarps][3][RS]
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* acc = sm + (size_t)wid * 3 * RS;
  for (int i = lane * 4; i < 3 * RS; i += 128) *reinterpret_cast<float4*>(acc + i) = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncwarp();
  const bool has_r = dresid != nullptr;
  const int r0 = blockIdx.x * kLnBwdRowsPerBlock;
  const int r_end = min(r0 + kLnBwdRowsPerBlock, rows);
  uint4 cy[NCH], cx[NCH], cr[NCH];
  auto load = [&](int r, uint4* gy, uint4* gx, uint4* gr) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < C) {
        gy[c] = *reinterpret_cast<const uint4*>(dy + (long)r * C + col);
        gx[c] = *reinterpret_cast<const uint4*>(x + (long)r * C + col);
        gr[c] = has_r ? *reinterpret_cast<const uint4*>(dresid + (long)r * C + col) : make_uint4(0, 0, 0, 0);
      }
    }
  };
  int r = r0 + wid;
  if (r < r_end) load(r, cy, cx, cr);
  for (; r < r_end; r += kLnBwdWarps) {
    constexpr bool kPrefetch = NCH <= 3;  // larger rows keep enough bytes in flight without it
    uint4 ny[NCH], nx[NCH], nr[NCH];
    if (kPrefetch && r + kLnBwdWarps < r_end) load(r + kLnBwdWarps, ny, nx, nr);
    const float mu = mean[r], rs = rstd[r];
    float s1 = 0.f, s2 = 0.f;
    // pass 1: row statistics of g*w and g*w*xhat, plus the column accumulators
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < C) {
        float g[8], xv[8], wv[8], rv[8];
        unpack8(cy[c], g);
        unpack8(cx[c], xv);
        ld8(w + col, wv);  // 1.5-6 KB of weights: L1-resident across rows
        // accumulator rows are lane-interleaved (float4 (c, h) of lane l at ((2c+h)*32+l)*4), so a
        // warp's float4 accesses are contiguous 512-byte runs without bank conflicts
        float4* aw = reinterpret_cast<float4*>(acc) + (2 * c) * 32 + lane;
        float4* ab = reinterpret_cast<float4*>(acc + RS) + (2 * c) * 32 + lane;
        float4 w0 = aw[0], w1 = aw[32], b0 = ab[0], b1 = ab[32];
        float dwv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float dbv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = (xv[j] - mu) * rs;
          const float gw = g[j] * wv[j];
          s1 += gw;
          s2 += gw * xh;
          dwv[j] += g[j] * xh;
          dbv[j] += g[j];
        }
        aw[0] = make_float4(dwv[0], dwv[1], dwv[2], dwv[3]);
        aw[32] = make_float4(dwv[4], dwv[5], dwv[6], dwv[7]);
        ab[0] = make_float4(dbv[0], dbv[1], dbv[2], dbv[3]);
        ab[32] = make_float4(dbv[4], dbv[5], dbv[6], dbv[7]);
        if (part_r) {
          unpack8(cr[c], rv);
          float4* ar = reinterpret_cast<float4*>(acc + 2 * RS) + (2 * c) * 32 + lane;
          float4 r0v = ar[0], r1v = ar[32];
          ar[0] = make_float4(r0v.x + rv[0], r0v.y + rv[1], r0v.z + rv[2], r0v.w + rv[3]);
          ar[32] = make_float4(r1v.x + rv[4], r1v.y + rv[5], r1v.z + rv[6], r1v.w + rv[7]);
        }
      }
    }
    const float m1 = warp_sum(s1) / C, m2 = warp_sum(s2) / C;
    // pass 2: dx from the registers
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < C) {
        float g[8], xv[8], wv[8], rv[8], o[8];
        unpack8(cy[c], g);
        unpack8(cx[c], xv);
        ld8(w + col, wv);
        unpack8(cr[c], rv);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = rs * (g[j] * wv[j] - m1 - (xv[j] - mu) * rs * m2) + rv[j];
        st8(dx + (long)r * C + col, o);
      }
    }
    if (kPrefetch) {
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        cy[c] = ny[c];
        cx[c] = nx[c];
        cr[c] = nr[c];
      }
    } else if (r + kLnBwdWarps < r_end) {
      load(r + kLnBwdWarps, cy, cx, cr);
    }
  }
  __syncthreads();
  // combine the warps of this block in warp order
  const int narr = part_r ? 3 : 2;
  for (int i = threadIdx.x; i < narr * RS; i += blockDim.x) {
    // undo the lane interleave: index j within a row is ((2c+h)*32 + lane)*4 + e
    const int a = i / RS, j = i - a * RS;
    const int e = j & 3, lane_j = (j >> 2) & 31, ch = j >> 7;  // ch = 2c + h
    const int col = ((ch >> 1) * 32 + lane_j) * 8 + (ch & 1) * 4 + e;
    if (col >= C) continue;
    float t = 0.f;
    for (int k = 0; k < kLnBwdWarps; ++k) t += sm[(size_t)k * 3 * RS + i];
    float* dst = a == 0 ? part_w : (a == 1 ? part_b : part_r);
    dst[(long)blockIdx.x * C + col] = t;
  }
}

// out[col] = (accumulate ? out[col] : 0) + sum_{k=0..nparts-1} part[k, col].
// Block = 32 columns x 32 partial-lanes: lane k sums partials k, k+32, ...
// (coalesced 128-byte rows), then the lane sums are combined in lane order - a
// fixed order, so the result is deterministic.  blockIdx.y picks one of up to
// three (part, out) pairs, so several reductions share a launch.
constexpr int kColsumLanes = 32;
struct ColsumJobs {
  const float* part[3];
  float* out[3];
};
__global__ void __launch_bounds__(32 * kColsumLanes)
    colsum_partials_kernel(ColsumJobs jobs, int nparts, int C, int accumulate) {
  __shared__ float sm[kColsumLanes][33];
  const float* part = jobs.part[blockIdx.y];
  float* out = jobs.out[blockIdx.y];
  const int cl = threadIdx.x & 31, kl = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + cl;
  float s = 0.f;
  if (col < C)
    for (int k = kl; k < nparts; k += kColsumLanes) s += part[(long)k * C + col];
  sm[kl][cl] = s;
  __syncthreads();
  if (kl == 0 && col < C) {
    float t = sm[0][cl];
#pragma unroll
    for (int i = 1; i < kColsumLanes; ++i) t += sm[i][cl];
    out[col] = accumulate ? out[col] + t : t;
  }
}

static inline void launch_colsum_multi(const ColsumJobs& jobs, int njobs, int nparts, int C, int accumulate,
                                       cudaStream_t st) {
  dim3 grid((C + 31) / 32, njobs);
  colsum_partials_kernel<<<grid, 32 * kColsumLanes, 0, st>>>(jobs, nparts, C, accumulate);
}

static inline void launch_colsum(const float* part, int nparts, int C, float* out, int accumulate,
                                 cudaStream_t st) {
  ColsumJobs j{};
  j.part[0] = part;
  j.out[0] = out;
  launch_colsum_multi(j, 1, nparts, C, accumulate, st);
}

// Bias gradient stage 1: partial column sums of a bf16 [rows, N] matrix over
// blocks of kColRows rows.  Thread layout: 32 column groups of 8 x 8 row lanes.
constexpr int kColRows = 128;
__global__ void __launch_bounds__(256)
    colsum_bf16_stage1(const bf16* __restrict__ g, long ld, int rows, int N, float* __restrict__ part) {
  __shared__ float sm[8][256 + 8];
  const int cg = threadIdx.x & 31, rl = threadIdx.x >> 5;
  const int col = blockIdx.x * 256 + cg * 8;
  const int r0 = blockIdx.y * kColRows;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (col < N) {
    for (int r = r0 + rl; r < min(r0 + kColRows, rows); r += 8) {
      float v[8];
      ld8(g + (long)r * ld + col, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += v[j];
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) sm[rl][cg * 8 + j] = acc[j];
  __syncthreads();
  const int c = threadIdx.x;
  if (blockIdx.x * 256 + c < N) {
    float s = 0.f;
    for (int k = 0; k < 8; ++k) s += sm[k][c];
    part[(long)blockIdx.y * N + blockIdx.x * 256 + c] = s;
  }
}

// ------------------------------------------------------------------ host
static int ln_chunks(int C) {
  TORCH_CHECK(C % 8 == 0 && C <= 2048, "layernorm: C must be a multiple of 8 and <= 2048, got ", C);
  return (C + 255) / 256;
}

std::vector<torch::Tensor> layernorm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor b, double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "layernorm_fwd: x");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "layernorm_fwd: w/b bf16");
  c10::cuda::CUDAGuard guard(x.device());
  const int C = (int)x.size(-1);
  const int rows = (int)(x.numel() / C);
  auto y = torch::empty_like(x);
  auto mean = torch::empty({rows}, x.options().dtype(at::kFloat));
  auto rstd = torch::empty({rows}, x.options().dtype(at::kFloat));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int threads = 256;
  const long warps = (rows + 1) / 2;  // two rows per warp
  const int blocks = (int)((warps * 32 + threads - 1) / threads);
  const int nch = ln_chunks(C);
  auto* xp = reinterpret_cast<const bf16*>(x.data_ptr());
  auto* wp = reinterpret_cast<const bf16*>(w.data_ptr());
  auto* bp = reinterpret_cast<const bf16*>(b.data_ptr());
  auto* yp = reinterpret_cast<bf16*>(y.data_ptr());
#define LNF(NC) ln_fwd_kernel<NC><<<blocks, threads, 0, st>>>(xp, wp, bp, yp, mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, C, (float)eps)
  switch (nch) {
    case 1: LNF(1); break;
    case 2: LNF(2); break;
    case 3: LNF(3); break;
    case 4: LNF(4); break;
    case 5: case 6: LNF(6); break;
    case 7: case 8: LNF(8); break;
    default: TORCH_CHECK(false, "layernorm: C too large");
  }
#undef LNF
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {y, mean, rstd};
}

// Returns dx; writes dw, db (fp32 [C]) - accumulating when requested - and, when
// `dres_sum` is given, the column sums of dresid (the bias gradient of the layer
// whose output gradient dresid is), so that bias gradient costs no extra pass.
torch::Tensor layernorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor mean,
                            torch::Tensor rstd, c10::optional<torch::Tensor> dresid, torch::Tensor dw,
                            torch::Tensor db, bool accumulate, c10::optional<torch::Tensor> dres_sum) {
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous() && dy.scalar_type() == at::kBFloat16, "layernorm_bwd: dy/x");
  TORCH_CHECK(dw.scalar_type() == at::kFloat && db.scalar_type() == at::kFloat, "layernorm_bwd: dw/db fp32");
  c10::cuda::CUDAGuard guard(x.device());
  const int C = (int)x.size(-1);
  const int rows = (int)(x.numel() / C);
  auto dx = torch::empty_like(x);
  const int nblk = (rows + kLnBwdRowsPerBlock - 1) / kLnBwdRowsPerBlock;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const bf16* dr = nullptr;
  if (dresid && dresid->defined()) {
    TORCH_CHECK(dresid->is_contiguous() && dresid->numel() == x.numel() && dresid->scalar_type() == at::kBFloat16,
                "layernorm_bwd: dresid");
    dr = reinterpret_cast<const bf16*>(dresid->data_ptr());
  }
  const bool rsum = dres_sum && dres_sum->defined();
  TORCH_CHECK(!rsum || (dr && dres_sum->scalar_type() == at::kFloat && dres_sum->numel() == C &&
                        dres_sum->is_contiguous()),
              "layernorm_bwd: dres_sum needs dresid and an fp32 [C] output");
  auto part = torch::empty({rsum ? 3 : 2, nblk, C}, x.options().dtype(at::kFloat));
  const int nch = ln_chunks(C);
  auto* dyp = reinterpret_cast<const bf16*>(dy.data_ptr());
  auto* xp = reinterpret_cast<const bf16*>(x.data_ptr());
  auto* wp = reinterpret_cast<const bf16*>(w.data_ptr());
  auto* dxp = reinterpret_cast<bf16*>(dx.data_ptr());
  float* pw = part.data_ptr<float>();
  float* pb = pw + (long)nblk * C;
  float* pr = rsum ? pb + (long)nblk * C : nullptr;
#define LNB(NC)                                                                                          \
  {                                                                                                      \
    auto k = ln_bwd_kernel<NC>;                                                                          \
    const size_t smem = ln_bwd_smem(NC);                                                                 \
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    k<<<nblk, kLnBwdWarps * 32, smem, st>>>(dyp, xp, wp, mean.data_ptr<float>(), rstd.data_ptr<float>(), dr, dxp, pw, pb, pr, rows, C); \
  }
  switch (nch) {
    case 1: LNB(1); break;
    case 2: LNB(2); break;
    case 3: LNB(3); break;
    case 4: LNB(4); break;
    case 5: case 6: LNB(6); break;
    case 7: case 8: LNB(8); break;
    default: TORCH_CHECK(false, "layernorm_bwd: C too large");
  }
#undef LNB
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  ColsumJobs jobs{};
  jobs.part[0] = pw;
  jobs.out[0] = dw.data_ptr<float>();
  jobs.part[1] = pb;
  jobs.out[1] = db.data_ptr<float>();
  if (rsum) {
    jobs.part[2] = pr;
    jobs.out[2] = dres_sum->data_ptr<float>();
  }
  launch_colsum_multi(jobs, rsum ? 3 : 2, nblk, C, accumulate ? 1 : 0, st);
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dx;
}

// db[N] (+)= column sums of g [rows, N] (bf16), deterministic.
void bias_grad(torch::Tensor g, torch::Tensor db, bool accumulate) {
  TORCH_CHECK(g.dim() == 2 && g.stride(1) == 1 && g.scalar_type() == at::kBFloat16, "bias_grad: g");
  TORCH_CHECK(db.scalar_type() == at::kFloat && db.is_contiguous(), "bias_grad: db");
  c10::cuda::CUDAGuard guard(g.device());
  const int rows = (int)g.size(0), N = (int)g.size(1);
  TORCH_CHECK(N % 8 == 0 && g.stride(0) % 8 == 0, "bias_grad: N must be a multiple of 8");
  const int rb = (rows + kColRows - 1) / kColRows;
  auto part = torch::empty({rb, N}, g.options().dtype(at::kFloat));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  dim3 grid((N + 255) / 256, rb);
  colsum_bf16_stage1<<<grid, 256, 0, st>>>(reinterpret_cast<const bf16*>(g.data_ptr()), g.stride(0), rows, N,
                                           part.data_ptr<float>());
  launch_colsum(part.data_ptr<float>(), rb, N, db.data_ptr<float>(), accumulate ? 1 : 0, st);
  count_launch(2);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

DTB_DEFINE_STATUS_READER(status_layernorm)

}  // namespace dtb

// ============================================================================
// dtb_layernorm_bwd_noalloc: allocation-free LayerNorm backward (C entry point)
// ============================================================================
// This entry point has no counterpart in the reference project.  Declaration,
// return codes, limits and rules: dtb_noalloc.h (included so the compiler checks
// this definition against it).
//
// What it computes: exactly what layernorm_bwd() above computes - dx (bf16),
// plus dw and db (fp32, written or accumulated) - with the same kernels and the
// same deterministic two-stage reduction.  The difference is where the per-block
// partial sums live: instead of a workspace from the caching allocator they go
// to the file-scope device array below, so nothing is allocated.
constexpr long kLnNoAllocScratchFloats = DTB_LN_NOALLOC_SCRATCH_FLOATS;

// The scratch array itself (one copy per device that loads this library).  In
// host code its name is only a host-side stand-in for the symbol: kernels get the
// device address that cudaGetSymbolAddress returns.
static __device__ __align__(256) float g_ln_noalloc_scratch[kLnNoAllocScratchFloats];

namespace {

constexpr int kNoAllocMaxDevices = 64;

struct ScratchEntry {
  CUcontext ctx;  // context the address belongs to
  float* ptr;
};
std::mutex g_noalloc_mu;
ScratchEntry g_noalloc_scratch[kNoAllocMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (CtxGetCurrentFn) nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  return fn;
}

// Device address of the scratch array in the current device's context.  Looked up
// with cudaGetSymbolAddress once per device and cached together with the context
// handle; a different context on the device (after cudaDeviceReset, say) is looked
// up again instead of reusing an address that belonged to the old one.
int noalloc_scratch(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return DTB_NOALLOC_SETUP_FAILED;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  CtxGetCurrentFn get = ctx_get_current();
  CUcontext ctx = nullptr;
  if (get) get(&ctx);
  ScratchEntry& e = g_noalloc_scratch[dev];
  if (e.ptr == nullptr || ctx == nullptr || e.ctx != ctx) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_ln_noalloc_scratch);
    if (err != cudaSuccess || p == nullptr) {
      std::fprintf(stderr, "dtb_layernorm_bwd_noalloc: cudaGetSymbolAddress failed on device %d: %s\n", dev,
                   cudaGetErrorString(err));
      return DTB_NOALLOC_SETUP_FAILED;
    }
    if (get && ctx == nullptr) get(&ctx);  // the lookup bound the primary context
    e.ptr = static_cast<float*>(p);
    e.ctx = ctx;
  }
  *out = e.ptr;
  return DTB_NOALLOC_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" __attribute__((visibility("default"))) int dtb_layernorm_bwd_noalloc(
    const void* dy, const void* x, const void* w, const float* mean, const float* rstd, const void* dresid,
    void* dx, float* dw, float* db, int rows, int C, int accumulate, cudaStream_t stream) {
  using namespace dtb;
  if (!dy || !x || !w || !mean || !rstd || !dx || !dw || !db || rows <= 0 || C <= 0 || C % 8 != 0 || C > 2048 ||
      !aligned16(dy) || !aligned16(x) || !aligned16(w) || !aligned16(dx) || (dresid && !aligned16(dresid)))
    return DTB_NOALLOC_BAD_ARGUMENT;
  const long nblk = (rows + kLnBwdRowsPerBlock - 1) / kLnBwdRowsPerBlock;
  const long need = 2 * nblk * (long)C;
  if (need > kLnNoAllocScratchFloats) {
    std::fprintf(stderr,
                 "dtb_layernorm_bwd_noalloc: rows=%d, C=%d needs %ld scratch floats (2 * ceil(rows / %d) * C), "
                 "more than the fixed %ld\n",
                 rows, C, need, kLnBwdRowsPerBlock, kLnNoAllocScratchFloats);
    return DTB_NOALLOC_TOO_LARGE;
  }
  // an error left by earlier work is the caller's, not this call's: report it without clearing it
  if (cudaPeekAtLastError() != cudaSuccess) return DTB_NOALLOC_PRIOR_ERROR;
  float* scratch = nullptr;
  if (noalloc_scratch(&scratch) != DTB_NOALLOC_OK) return DTB_NOALLOC_SETUP_FAILED;
  float* pw = scratch;
  float* pb = scratch + nblk * C;
  const int nch = (C + 255) / 256;
  auto* dyp = static_cast<const bf16*>(dy);
  auto* xp = static_cast<const bf16*>(x);
  auto* wp = static_cast<const bf16*>(w);
  auto* drp = static_cast<const bf16*>(dresid);
  auto* dxp = static_cast<bf16*>(dx);
#define DTB_LNB_NOALLOC(NC)                                                                                       \
  {                                                                                                               \
    auto k = ln_bwd_kernel<NC>;                                                                                   \
    const size_t smem = ln_bwd_smem(NC);                                                                          \
    if (smem > 48 * 1024 && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=     \
                                cudaSuccess) {                                                                    \
      cudaGetLastError();                                                                                         \
      return DTB_NOALLOC_LAUNCH_FAILED;                                                                           \
    }                                                                                                             \
    k<<<(unsigned)nblk, kLnBwdWarps * 32, smem, stream>>>(dyp, xp, wp, mean, rstd, drp, dxp, pw, pb, nullptr, rows, \
                                                          C);                                                     \
  }
  switch (nch) {
    case 1: DTB_LNB_NOALLOC(1); break;
    case 2: DTB_LNB_NOALLOC(2); break;
    case 3: DTB_LNB_NOALLOC(3); break;
    case 4: DTB_LNB_NOALLOC(4); break;
    case 5: case 6: DTB_LNB_NOALLOC(6); break;
    default: DTB_LNB_NOALLOC(8); break;
  }
#undef DTB_LNB_NOALLOC
  // the column sums must not run on partials the first kernel never wrote
  if (cudaGetLastError() != cudaSuccess) return DTB_NOALLOC_LAUNCH_FAILED;
  ColsumJobs jobs{};
  jobs.part[0] = pw;
  jobs.out[0] = dw;
  jobs.part[1] = pb;
  jobs.out[1] = db;
  launch_colsum_multi(jobs, 2, (int)nblk, C, accumulate ? 1 : 0, stream);
  if (cudaGetLastError() != cudaSuccess) return DTB_NOALLOC_LAUNCH_FAILED;
  return DTB_NOALLOC_OK;
}


