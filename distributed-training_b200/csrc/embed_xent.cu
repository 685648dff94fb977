// Token/position embedding and softmax cross-entropy kernels.
//
// Embedding (dtrain/autograd.py:199-204, dtrain/nn.py:133): forward gathers
// tok[idx] + pos[t]; the backward is a scatter-add with repeated indices.  The
// reference uses np.add.at; here the scatter is made deterministic without float
// atomics: the host sorts the flat token ids stably (ties keep position order),
// and one warp per vocabulary row sums its positions' gradient rows in that order.
//
// Cross-entropy (dtrain/autograd.py:250-266): mean over rows of logsumexp(z) - z[t].
// The forward keeps the per-row logsumexp; the backward rewrites the logits buffer
// in place with (softmax - onehot) * g / n, so the V-wide gradient needs no new
// allocation.  The mean over rows is a fixed-order reduction.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace dtb {

__device__ __forceinline__ void ld8f(const bf16* p, float* v) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ void st8f(bf16* p, const float* v) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

// ------------------------------------------------------------------ embedding
__global__ void embed_fwd_kernel(const int64_t* __restrict__ idx, const bf16* __restrict__ tok,
                                 const bf16* __restrict__ pos, bf16* __restrict__ out, long ntok, int T, int C, int V,
                                 int* __restrict__ bad) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;  // one thread per 8 channels
  const int per_row = C / 8;
  if (i >= ntok * per_row) return;
  const long r = i / per_row;
  const int c = (int)(i % per_row) * 8;
  int64_t t = idx[r];
  if (t < 0 || t >= V) {  // out-of-range token: record and emit zeros instead of reading out of bounds
    if (c == 0) atomicExch(bad, 1);
    float z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    st8f(out + r * C + c, z);
    return;
  }
  float a[8], b[8];
  ld8f(tok + t * C + c, a);
  ld8f(pos + (long)(r % T) * C + c, b);
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] += b[j];
  st8f(out + r * C + c, a);
}

// ---------------------------------------------------------- stable id sort
// LSD radix sort of the token ids with 8-bit digits (two passes for vocabularies
// up to 65536), carrying each token's position.  Every pass is three small
// kernels: per-block digit histograms, one scan that turns them into each
// block's first output slot per digit, and a scatter that ranks equal digits
// inside a block in position order (warp match + per-warp counts), so the sort
// is stable and its output depends only on the ids: equal ids stay in position
// order, which fixes the summation order of the embedding gradient below.
constexpr int kSortBlock = 1024;  // elements (and threads) per block
constexpr int kSortBins = 256;

__device__ __forceinline__ int sort_key(long i, long n, const int64_t* key64, const int* key32, int vclamp) {
  if (i >= n) return -1;
  long k = key64 ? key64[i] : (long)key32[i];
  return (k < 0 || k > vclamp) ? vclamp : (int)k;  // ids outside [0, V) sort last and match no row
}

__global__ void __launch_bounds__(kSortBlock)
    sort_hist_kernel(const int64_t* key64, const int* key32, long n, int vclamp, int shift, int* ghist) {
  __shared__ int h[kSortBins];
  for (int k = threadIdx.x; k < kSortBins; k += blockDim.x) h[k] = 0;
  __syncthreads();
  const int key = sort_key((long)blockIdx.x * kSortBlock + threadIdx.x, n, key64, key32, vclamp);
  if (key >= 0) atomicAdd(&h[(key >> shift) & 255], 1);
  __syncthreads();
  for (int k = threadIdx.x; k < kSortBins; k += blockDim.x) ghist[(long)blockIdx.x * kSortBins + k] = h[k];
}

// goff[b][k] = (number of keys with digit < k) + (keys with digit k in blocks < b)
__global__ void __launch_bounds__(kSortBins) sort_scan_kernel(const int* ghist, int nblk, int* goff) {
  __shared__ int tot[kSortBins];
  const int k = threadIdx.x;
  int t = 0;
  for (int b = 0; b < nblk; ++b) t += ghist[(long)b * kSortBins + k];
  tot[k] = t;
  __syncthreads();
  int base = 0;
  for (int j = 0; j < k; ++j) base += tot[j];
  for (int b = 0; b < nblk; ++b) {
    goff[(long)b * kSortBins + k] = base;
    base += ghist[(long)b * kSortBins + k];
  }
}

template <bool FINAL>
__global__ void __launch_bounds__(kSortBlock)
    sort_scatter_kernel(const int64_t* key64, const int* key32, const int* val_in, long n, int vclamp, int shift,
                        const int* goff, int* key_out, int* val_out, int64_t* key_out64, int64_t* val_out64) {
  constexpr int kWarps = kSortBlock / 32;
  __shared__ int wcount[kWarps][kSortBins];
  for (int i = threadIdx.x; i < kWarps * kSortBins; i += blockDim.x) (&wcount[0][0])[i] = 0;
  __syncthreads();
  const long i = (long)blockIdx.x * kSortBlock + threadIdx.x;
  const int key = sort_key(i, n, key64, key32, vclamp);
  const int digit = key >= 0 ? (key >> shift) & 255 : kSortBins;  // kSortBins: no element
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned same = __match_any_sync(0xffffffffu, digit);
  const int rank_in_warp = __popc(same & ((1u << lane) - 1u));
  if (digit < kSortBins && rank_in_warp == 0) wcount[warp][digit] = __popc(same);
  __syncthreads();
  // exclusive scan of every digit's count over the warps (in warp order)
  for (int k = threadIdx.x; k < kSortBins; k += blockDim.x) {
    int run = 0;
    for (int w = 0; w < kWarps; ++w) {
      const int c = wcount[w][k];
      wcount[w][k] = run;
      run += c;
    }
  }
  __syncthreads();
  if (digit < kSortBins) {
    const long dst = goff[(long)blockIdx.x * kSortBins + digit] + wcount[warp][digit] + rank_in_warp;
    const int val = val_in ? val_in[i] : (int)i;
    if (FINAL) {
      key_out64[dst] = key;
      val_out64[dst] = val;
    } else {
      key_out[dst] = key;
      val_out[dst] = val;
    }
  }
}

// Stable sort of idx (int64 [n], values in [0, V)): returns (sorted ids, positions) as int64.
std::vector<torch::Tensor> sort_ids(torch::Tensor idx, int64_t V) {
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == at::kLong && idx.is_contiguous(), "sort_ids: int64 CUDA ids");
  TORCH_CHECK(V >= 1 && V < (1L << 24), "sort_ids: vocabulary must be below 2^24");
  TORCH_CHECK(idx.numel() < (1L << 31), "sort_ids: too many ids");
  c10::cuda::CUDAGuard guard(idx.device());
  const long n = idx.numel();
  auto opt32 = idx.options().dtype(at::kInt);
  auto sorted = torch::empty({n}, idx.options());
  auto perm = torch::empty({n}, idx.options());
  if (n == 0) return {sorted, perm};
  const int nblk = (int)((n + kSortBlock - 1) / kSortBlock);
  auto hist = torch::empty({2, (long)nblk * kSortBins}, opt32);
  auto ka = torch::empty({n}, opt32), va = torch::empty({n}, opt32);
  auto kb = torch::empty({n}, opt32), vb = torch::empty({n}, opt32);
  const int vclamp = (int)V;  // out-of-range ids become V
  int passes = 1;
  while (passes < 3 && (vclamp >> (8 * passes)) > 0) ++passes;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int64_t* k64 = idx.data_ptr<int64_t>();
  const int* kin = nullptr;
  const int* vin = nullptr;
  int* gh = hist[0].data_ptr<int>();
  int* go = hist[1].data_ptr<int>();
  for (int p = 0; p < passes; ++p) {
    const int shift = 8 * p;
    const bool last = p == passes - 1;
    int* kout = (p % 2 == 0) ? ka.data_ptr<int>() : kb.data_ptr<int>();
    int* vout = (p % 2 == 0) ? va.data_ptr<int>() : vb.data_ptr<int>();
    sort_hist_kernel<<<nblk, kSortBlock, 0, st>>>(p == 0 ? k64 : nullptr, kin, n, vclamp, shift, gh);
    sort_scan_kernel<<<1, kSortBins, 0, st>>>(gh, nblk, go);
    if (last)
      sort_scatter_kernel<true><<<nblk, kSortBlock, 0, st>>>(p == 0 ? k64 : nullptr, kin, vin, n, vclamp, shift, go,
                                                             nullptr, nullptr, sorted.data_ptr<int64_t>(),
                                                             perm.data_ptr<int64_t>());
    else
      sort_scatter_kernel<false><<<nblk, kSortBlock, 0, st>>>(p == 0 ? k64 : nullptr, kin, vin, n, vclamp, shift, go,
                                                              kout, vout, nullptr, nullptr);
    count_launch(3);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    kin = kout;
    vin = vout;
  }
  return {sorted, perm};
}

// dtok[v] = sum over sorted positions p in [lo(v), hi(v)) of dx[perm[p]]  (one warp per v)
__global__ void embed_bwd_tok_kernel(const int64_t* __restrict__ sorted_ids, const int64_t* __restrict__ perm,
                                     long ntok, const bf16* __restrict__ dx, float* __restrict__ dtok, int V, int C,
                                     int accumulate) {
  const long v = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (v >= V) return;
  // lower_bound(v) and lower_bound(v+1) in sorted_ids
  long lo = 0, hi = ntok;
  while (lo < hi) {
    long m = (lo + hi) >> 1;
    if (sorted_ids[m] < v) lo = m + 1; else hi = m;
  }
  const long beg = lo;
  hi = ntok;
  while (lo < hi) {
    long m = (lo + hi) >> 1;
    if (sorted_ids[m] <= v) lo = m + 1; else hi = m;
  }
  const long end = lo;
  float* out = dtok + v * C;
  for (int c = lane * 4; c < C; c += 128) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (long p = beg; p < end; ++p) {
      const bf16* s = dx + perm[p] * C + c;
      __nv_bfloat162 h0 = *reinterpret_cast<const __nv_bfloat162*>(s);
      __nv_bfloat162 h1 = *reinterpret_cast<const __nv_bfloat162*>(s + 2);
      float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
      acc.x += f0.x; acc.y += f0.y; acc.z += f1.x; acc.w += f1.y;
    }
    float4* o = reinterpret_cast<float4*>(out + c);
    if (accumulate) {
      float4 p = *o;
      acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
    }
    *o = acc;
  }
}

// dpos[t] = sum_b dx[b*T + t]  (fixed order over b)
__global__ void embed_bwd_pos_kernel(const bf16* __restrict__ dx, float* __restrict__ dpos, int B, int T, int C,
                                     int accumulate) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)T * C) return;
  const int t = (int)(i / C), c = (int)(i % C);
  float s = 0.f;
  for (int b = 0; b < B; ++b) s += bf2f(dx[((long)b * T + t) * C + c]);
  dpos[i] = accumulate ? dpos[i] + s : s;
}

// ------------------------------------------------------------------ cross-entropy
constexpr int kXentThreads = 512;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) { m = m2; s = s2; return; }
  if (m2 > m) { s = s * __expf(m - m2) + s2; m = m2; }
  else { s = s + s2 * __expf(m2 - m); }
}

// One block per row: lse[row] = log(sum(exp(z))), loss[row] = lse - z[target].
__global__ void __launch_bounds__(kXentThreads)
    xent_fwd_kernel(const bf16* __restrict__ logits, long ld, const int64_t* __restrict__ tgt, int V,
                    float* __restrict__ lse_out, float* __restrict__ loss_out, int vec_ok) {
  const long row = blockIdx.x;
  const bf16* z = logits + row * ld;
  float m = -INFINITY, s = 0.f;
  const int nvec = vec_ok ? V / 8 : 0;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float v[8];
    ld8f(z + i * 8, v);
    float lm = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) lm = fmaxf(lm, v[j]);
    float ls = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ls += __expf(v[j] - lm);
    online_merge(m, s, lm, ls);
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += blockDim.x) online_merge(m, s, bf2f(z[i]), 1.f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  __shared__ float sm_m[kXentThreads / 32], sm_s[kXentThreads / 32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { sm_m[w] = m; sm_s[w] = s; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm_m[0], S = sm_s[0];
    for (int k = 1; k < kXentThreads / 32; ++k) online_merge(M, S, sm_m[k], sm_s[k]);
    const float lse = M + __logf(S);
    lse_out[row] = lse;
    const int64_t t = tgt[row];
    loss_out[row] = (t >= 0 && t < V) ? lse - bf2f(z[t]) : 0.f;
  }
}

// 2^x on the special-function unit (PTX ex2.approx, ~2 ulp; 2^-inf = +0).  The
// arguments are (x - rowmax) * log2(e) <= 0, so no range handling is needed.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Streaming variant for 16-byte aligned rows: each thread walks its strided
// 8-column chunks four at a time (the next four loads are in flight while the
// current ones are reduced), takes the max of the 32 values, merges it into its
// running (max, sum) once - two exponentials per 32 elements instead of per 8 -
// and then spends one exp2 per element on (x - max) * log2(e).
constexpr int kXentRound = 4;
__global__ void __launch_bounds__(kXentThreads)
    xent_fwd_stream_kernel(const bf16* __restrict__ logits, long ld, const int64_t* __restrict__ tgt, int V,
                           float* __restrict__ lse_out, float* __restrict__ loss_out) {
  constexpr float kLog2e = 1.4426950408889634f;
  const long row = blockIdx.x;
  const bf16* z = logits + row * ld;
  const int nvec = V / 8;
  float m = -INFINITY, s = 0.f;
  uint4 cur[kXentRound];
  auto load = [&](int base, uint4* dst) {
#pragma unroll
    for (int k = 0; k < kXentRound; ++k) {
      const int i = base + k * kXentThreads;
      if (i < nvec) dst[k] = *reinterpret_cast<const uint4*>(z + (long)i * 8);
    }
  };
  constexpr int kStep = kXentRound * kXentThreads;
  int base = threadIdx.x;
  if (base < nvec) load(base, cur);
  for (; base < nvec; base += kStep) {
    uint4 nxt[kXentRound];
    if (base + kStep < nvec) load(base + kStep, nxt);
    float lm = -INFINITY;
#pragma unroll
    for (int k = 0; k < kXentRound; ++k) {
      if (base + k * kXentThreads < nvec) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&cur[k]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          lm = fmaxf(lm, fmaxf(f.x, f.y));
        }
      }
    }
    const float nb = -lm * kLog2e;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int k = 0; k < kXentRound; ++k) {
      if (base + k * kXentThreads < nvec) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&cur[k]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          s0 += ex2_approx(fmaf(f.x, kLog2e, nb));
          s1 += ex2_approx(fmaf(f.y, kLog2e, nb));
        }
      }
    }
    online_merge(m, s, lm, s0 + s1);
#pragma unroll
    for (int k = 0; k < kXentRound; ++k) cur[k] = nxt[k];
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += kXentThreads) online_merge(m, s, bf2f(z[i]), 1.f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  __shared__ float sm_m[kXentThreads / 32], sm_s[kXentThreads / 32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { sm_m[w] = m; sm_s[w] = s; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm_m[0], S = sm_s[0];
    for (int k = 1; k < kXentThreads / 32; ++k) online_merge(M, S, sm_m[k], sm_s[k]);
    const float lse = M + __logf(S);
    lse_out[row] = lse;
    const int64_t t = tgt[row];
    loss_out[row] = (t >= 0 && t < V) ? lse - bf2f(z[t]) : 0.f;
  }
}

// loss = mean(loss_rows) in a fixed order (single block).
__global__ void mean_kernel(const float* __restrict__ x, long n, float* __restrict__ out) {
  __shared__ double sm[1024];
  double s = 0.0;
  for (long i = threadIdx.x; i < n; i += blockDim.x) s += (double)x[i];
  sm[threadIdx.x] = s;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) sm[threadIdx.x] += sm[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[0] = (float)(sm[0] / (double)n);
}

// In place: z[row, j] <- (exp(z - lse) - [j == t]) * g / n     (g read from device memory)
__global__ void __launch_bounds__(kXentThreads)
    xent_bwd_kernel(bf16* __restrict__ logits, long ld, const int64_t* __restrict__ tgt, int V,
                    const float* __restrict__ lse, const float* __restrict__ gscale, float inv_n, int vec_ok) {
  const long row = blockIdx.x;
  bf16* z = logits + row * ld;
  const float L = lse[row];
  const float g = gscale[0] * inv_n;
  const int64_t t = tgt[row];
  const int nvec = vec_ok ? V / 8 : 0;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float v[8];
    ld8f(z + i * 8, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float p = __expf(v[j] - L);
      if (i * 8 + j == t) p -= 1.f;
      v[j] = p * g;
    }
    st8f(z + i * 8, v);
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += blockDim.x) {
    float p = __expf(bf2f(z[i]) - L);
    if (i == t) p -= 1.f;
    z[i] = f2bf(p * g);
  }
}

// ------------------------------------------------------------------ host
torch::Tensor embed_fwd(torch::Tensor idx, torch::Tensor tok, torch::Tensor pos, torch::Tensor bad_flag) {
  TORCH_CHECK(idx.scalar_type() == at::kLong && idx.is_contiguous() && idx.dim() == 2, "embed_fwd: idx [B,T] int64");
  TORCH_CHECK(tok.scalar_type() == at::kBFloat16 && pos.scalar_type() == at::kBFloat16, "embed_fwd: bf16 tables");
  c10::cuda::CUDAGuard guard(idx.device());
  const int B = (int)idx.size(0), T = (int)idx.size(1);
  const int V = (int)tok.size(0), C = (int)tok.size(1);
  TORCH_CHECK(C % 8 == 0 && pos.size(0) >= T && pos.size(1) == C, "embed_fwd: shapes");
  auto out = torch::empty({B, T, C}, tok.options());
  const long ntok = (long)B * T;
  const long work = ntok * (C / 8);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  embed_fwd_kernel<<<(unsigned)((work + 255) / 256), 256, 0, st>>>(
      idx.data_ptr<int64_t>(), reinterpret_cast<const bf16*>(tok.data_ptr()),
      reinterpret_cast<const bf16*>(pos.data_ptr()), reinterpret_cast<bf16*>(out.data_ptr()), ntok, T, C, V,
      bad_flag.data_ptr<int>());
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// idx [B*T] int64 token ids; dtok [V,C] fp32, dpos [>=T,C] fp32.  The ids are
// stably sorted by sort_ids() (this file's radix sort) so each vocabulary row sums
// its positions in increasing order.
void embed_bwd(torch::Tensor idx, torch::Tensor dx, torch::Tensor dtok, torch::Tensor dpos, int64_t B, int64_t T,
               bool accumulate) {
  TORCH_CHECK(dx.scalar_type() == at::kBFloat16 && dx.is_contiguous(), "embed_bwd: dx");
  TORCH_CHECK(dtok.scalar_type() == at::kFloat && dpos.scalar_type() == at::kFloat, "embed_bwd: fp32 grads");
  TORCH_CHECK(idx.numel() == B * T, "embed_bwd: B*T ids expected");
  c10::cuda::CUDAGuard guard(dx.device());
  const int V = (int)dtok.size(0), C = (int)dtok.size(1);
  auto sp = sort_ids(idx.reshape({-1}).contiguous(), V);
  const torch::Tensor& sorted_ids = sp[0];
  const torch::Tensor& perm = sp[1];
  TORCH_CHECK(C % 4 == 0, "embed_bwd: C % 4");
  const long ntok = B * T;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const long threads = (long)V * 32;
  embed_bwd_tok_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
      sorted_ids.data_ptr<int64_t>(), perm.data_ptr<int64_t>(), ntok, reinterpret_cast<const bf16*>(dx.data_ptr()),
      dtok.data_ptr<float>(), V, C, accumulate ? 1 : 0);
  const long n = T * (long)C;
  embed_bwd_pos_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(reinterpret_cast<const bf16*>(dx.data_ptr()),
                                                                    dpos.data_ptr<float>(), (int)B, (int)T, C,
                                                                    accumulate ? 1 : 0);
  count_launch(2);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Returns (loss scalar fp32 [1], lse fp32 [rows]).
std::vector<torch::Tensor> xent_fwd(torch::Tensor logits, torch::Tensor tgt) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1 && logits.scalar_type() == at::kBFloat16, "xent_fwd: logits");
  TORCH_CHECK(tgt.scalar_type() == at::kLong && tgt.numel() == logits.size(0), "xent_fwd: targets");
  c10::cuda::CUDAGuard guard(logits.device());
  const long rows = logits.size(0);
  const int V = (int)logits.size(1);
  const int vec_ok = (logits.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(logits.data_ptr()) & 15) == 0) ? 1 : 0;
  auto lse = torch::empty({rows}, logits.options().dtype(at::kFloat));
  auto lrow = torch::empty({rows}, logits.options().dtype(at::kFloat));
  auto loss = torch::empty({}, logits.options().dtype(at::kFloat));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto tg = tgt.contiguous();
  auto* zp = reinterpret_cast<const bf16*>(logits.data_ptr());
  if (vec_ok) {
    xent_fwd_stream_kernel<<<(unsigned)rows, kXentThreads, 0, st>>>(zp, logits.stride(0), tg.data_ptr<int64_t>(), V,
                                                                    lse.data_ptr<float>(), lrow.data_ptr<float>());
  } else {
    xent_fwd_kernel<<<(unsigned)rows, kXentThreads, 0, st>>>(zp, logits.stride(0), tg.data_ptr<int64_t>(), V,
                                                            lse.data_ptr<float>(), lrow.data_ptr<float>(), vec_ok);
  }
  mean_kernel<<<1, 1024, 0, st>>>(lrow.data_ptr<float>(), rows, loss.data_ptr<float>());
  count_launch(2);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {loss, lse};
}

// Cross-entropy forward (dtrain/autograd.py:250-266: mean over rows of lse - z[target])
// from the LM-head GEMM's softmax partials (EPI_LSE in gemm.cu):
// part[row, p] = (max, sum exp(x - max)) over column half-tile p of the bf16 logits.
// One warp per row merges its partials in a fixed order (lane-strided, then a fixed
// shuffle tree), so the result is deterministic; loss_row = lse - z[target].
__global__ void __launch_bounds__(256)
    xent_parts_kernel(const float2* __restrict__ part, int np, const bf16* __restrict__ logits, long ld,
                      const int64_t* __restrict__ tgt, int V, long rows, float* __restrict__ lse_out,
                      float* __restrict__ loss_out) {
  const long row = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float2* pr = part + row * np;
  float m = -INFINITY, s = 0.f;
  for (int p = lane; p < np; p += 32) {
    const float2 q = pr[p];
    online_merge(m, s, q.x, q.y);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  if (lane == 0) {
    const float lse = m + __logf(s);
    lse_out[row] = lse;
    const int64_t t = tgt[row];
    loss_out[row] = (t >= 0 && t < V) ? lse - bf2f(logits[row * ld + t]) : 0.f;
  }
}

// Returns (loss scalar fp32 [1], lse fp32 [rows]) from the head GEMM's partials.
std::vector<torch::Tensor> xent_from_parts(torch::Tensor part, torch::Tensor logits, torch::Tensor tgt) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1 && logits.scalar_type() == at::kBFloat16,
              "xent_from_parts: logits");
  TORCH_CHECK(part.dim() == 3 && part.size(2) == 2 && part.scalar_type() == at::kFloat && part.is_contiguous() &&
                  part.size(0) == logits.size(0),
              "xent_from_parts: partials must be [rows, np, 2] fp32");
  TORCH_CHECK(tgt.scalar_type() == at::kLong && tgt.numel() == logits.size(0), "xent_from_parts: targets");
  c10::cuda::CUDAGuard guard(logits.device());
  const long rows = logits.size(0);
  auto lse = torch::empty({rows}, logits.options().dtype(at::kFloat));
  auto lrow = torch::empty({rows}, logits.options().dtype(at::kFloat));
  auto loss = torch::empty({}, logits.options().dtype(at::kFloat));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto tg = tgt.contiguous();
  xent_parts_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(
      reinterpret_cast<const float2*>(part.data_ptr<float>()), (int)part.size(1),
      reinterpret_cast<const bf16*>(logits.data_ptr()), logits.stride(0), tg.data_ptr<int64_t>(),
      (int)logits.size(1), rows, lse.data_ptr<float>(), lrow.data_ptr<float>());
  mean_kernel<<<1, 1024, 0, st>>>(lrow.data_ptr<float>(), rows, loss.data_ptr<float>());
  count_launch(2);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {loss, lse};
}

void xent_bwd(torch::Tensor logits, torch::Tensor tgt, torch::Tensor lse, torch::Tensor gscale) {
  c10::cuda::CUDAGuard guard(logits.device());
  const long rows = logits.size(0);
  const int V = (int)logits.size(1);
  TORCH_CHECK(gscale.scalar_type() == at::kFloat && gscale.numel() == 1, "xent_bwd: gscale");
  auto tg = tgt.contiguous();
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  xent_bwd_kernel<<<(unsigned)rows, kXentThreads, 0, st>>>(reinterpret_cast<bf16*>(logits.data_ptr()),
                                                          logits.stride(0), tg.data_ptr<int64_t>(), V,
                                                          lse.data_ptr<float>(), gscale.data_ptr<float>(),
                                                          1.0f / (float)rows,
                                                          (logits.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(logits.data_ptr()) & 15) == 0) ? 1 : 0);
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

DTB_DEFINE_STATUS_READER(status_embed_xent)

}  // namespace dtb
