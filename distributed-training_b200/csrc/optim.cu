// Flat-buffer optimizer kernels: AdamW, deterministic squared grad norm, casts.
//
// AdamW is the update of dtrain/optim.py:21-33 (decoupled decay first, then the
// moments, then the bias-corrected step), with the per-step constants folded on
// the host (adamw_elem in common.cuh: one square root and one division per
// element, the form torch.optim.AdamW uses):
//   p *= 1 - lr*wd ; m = b1*m + (1-b1)*g ; v = b2*v + (1-b2)*g*g
//   p -= (lr/b1t) * m / (sqrt(v)/sqrt(b2t) + eps)
// The bit-exact reference order lives in the fp64 host path (ops/optim.py).  It
// runs over one flat fp32 master buffer (all parameters, or a ZeRO shard), and also
// refreshes the bf16 working copy the GEMMs read.  Global-norm clipping
// (dtrain/optim.py:49-52, dtrain/train.py:155-158) is applied on the device: the
// kernel reads the squared norm produced by grad_sqnorm and computes the clip
// factor itself, so no host synchronisation sits between backward and the update.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace dtb {

__device__ __forceinline__ float clip_factor(const double* sq, float max_norm) {
  if (sq == nullptr || max_norm <= 0.f) return 1.f;
  const double n = sqrt(*sq);
  if (n <= (double)max_norm || n == 0.0) return 1.f;
  return (float)((double)max_norm / (n + 1e-6));
}

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, bf16* __restrict__ p16, long n, AdamConsts ak,
                             const double* __restrict__ sq, float max_norm) {
  const float cs = clip_factor(sq, max_norm);
  const long stride = (long)gridDim.x * blockDim.x * 4;
  for (long i = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < n; i += stride) {
    if (i + 4 <= n) {
      float4 pv = *reinterpret_cast<float4*>(p + i);
      const float4 gv = *reinterpret_cast<const float4*>(g + i);
      float4 mv = *reinterpret_cast<float4*>(m + i);
      float4 vv = *reinterpret_cast<float4*>(v + i);
      adamw_elem(pv.x, gv.x * cs, mv.x, vv.x, ak);
      adamw_elem(pv.y, gv.y * cs, mv.y, vv.y, ak);
      adamw_elem(pv.z, gv.z * cs, mv.z, vv.z, ak);
      adamw_elem(pv.w, gv.w * cs, mv.w, vv.w, ak);
      *reinterpret_cast<float4*>(p + i) = pv;
      *reinterpret_cast<float4*>(m + i) = mv;
      *reinterpret_cast<float4*>(v + i) = vv;
      if (p16) {
        uint2 u;
        u.x = pack_bf16x2(pv.x, pv.y);
        u.y = pack_bf16x2(pv.z, pv.w);
        *reinterpret_cast<uint2*>(p16 + i) = u;
      }
    } else {
      for (long k = i; k < n; ++k) {
        float pp = p[k], mm = m[k], vv2 = v[k];
        adamw_elem(pp, g[k] * cs, mm, vv2, ak);
        p[k] = pp;
        m[k] = mm;
        v[k] = vv2;
        if (p16) p16[k] = f2bf(pp);
      }
    }
  }
}

constexpr int kNormThreads = 256;
constexpr int kNormBlocks = 592;  // 4 x 148 SMs; fixed so the reduction order never changes

// Stage 1: block b sums g[i]^2 (as fp64) over its contiguous slice, tree-reduced in a fixed order.
__global__ void __launch_bounds__(kNormThreads)
    sqnorm_stage1(const float* __restrict__ g, long n, double* __restrict__ part) {
  __shared__ double sm[kNormThreads];
  const long chunk = (n + gridDim.x - 1) / gridDim.x;
  const long lo = (long)blockIdx.x * chunk;
  const long hi = min(n, lo + chunk);
  double s = 0.0;
  for (long i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const double x = (double)g[i];
    s += x * x;
  }
  sm[threadIdx.x] = s;
  __syncthreads();
  for (int o = kNormThreads / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) sm[threadIdx.x] += sm[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = sm[0];
}

// Stage 2: out[0] = sum of the partials (fixed tree order), optionally scaled.
__global__ void __launch_bounds__(kNormThreads)
    sqnorm_stage2(const double* __restrict__ part, int np, double* __restrict__ out, double scale) {
  __shared__ double sm[kNormThreads];
  double s = 0.0;
  for (int i = threadIdx.x; i < np; i += blockDim.x) s += part[i];
  sm[threadIdx.x] = s;
  __syncthreads();
  for (int o = kNormThreads / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) sm[threadIdx.x] += sm[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[0] = sm[0] * scale;
}

__global__ void cast_f32_bf16_kernel(const float* __restrict__ x, bf16* __restrict__ y, long n) {
  const long stride = (long)gridDim.x * blockDim.x;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) y[i] = f2bf(x[i]);
}

__global__ void scale_f32_kernel(float* __restrict__ x, long n, float s) {
  const long stride = (long)gridDim.x * blockDim.x;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) x[i] *= s;
}

// ------------------------------------------------------------------ host
static int grid_for(long n, int per_thread, int threads = 256) {
  long b = (n / per_thread + threads - 1) / threads;
  return (int)std::max<long>(1, std::min<long>(b, 148L * 16));
}

void adamw_step(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, c10::optional<torch::Tensor> p16,
                double lr, double b1, double b2, double eps, double wd, int64_t t, c10::optional<torch::Tensor> sq,
                double max_norm) {
  TORCH_CHECK(p.scalar_type() == at::kFloat && g.scalar_type() == at::kFloat && m.scalar_type() == at::kFloat &&
                  v.scalar_type() == at::kFloat,
              "adamw_step: fp32 buffers expected");
  TORCH_CHECK(p.is_contiguous() && g.is_contiguous() && m.is_contiguous() && v.is_contiguous(), "adamw: contiguous");
  const long n = p.numel();
  TORCH_CHECK(g.numel() == n && m.numel() == n && v.numel() == n, "adamw_step: size mismatch");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(p.data_ptr()) & 15) == 0 && (reinterpret_cast<uintptr_t>(g.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(m.data_ptr()) & 15) == 0 && (reinterpret_cast<uintptr_t>(v.data_ptr()) & 15) == 0,
              "adamw_step: 16-byte aligned buffers expected");
  c10::cuda::CUDAGuard guard(p.device());
  bf16* q = nullptr;
  if (p16 && p16->defined()) {
    TORCH_CHECK(p16->scalar_type() == at::kBFloat16 && p16->numel() == n && p16->is_contiguous() &&
                    (reinterpret_cast<uintptr_t>(p16->data_ptr()) & 7) == 0,
                "adamw_step: bf16 copy");
    q = reinterpret_cast<bf16*>(p16->data_ptr());
  }
  const double* sqp = nullptr;
  if (sq && sq->defined()) {
    TORCH_CHECK(sq->scalar_type() == at::kDouble && sq->numel() >= 1, "adamw_step: sq fp64");
    sqp = sq->data_ptr<double>();
  }
  if (n == 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  adamw_kernel<<<grid_for(n, 4), 256, 0, st>>>(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(),
                                              v.data_ptr<float>(), q, n, adam_consts(lr, b1, b2, eps, wd, t), sqp,
                                              (float)max_norm);
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out (fp64 [>=1]) = scale * sum(g^2), deterministic.
void grad_sqnorm(torch::Tensor g, torch::Tensor out, double scale) {
  TORCH_CHECK(g.scalar_type() == at::kFloat && g.is_contiguous(), "grad_sqnorm: fp32 contiguous");
  TORCH_CHECK(out.scalar_type() == at::kDouble, "grad_sqnorm: out fp64");
  c10::cuda::CUDAGuard guard(g.device());
  auto part = torch::empty({kNormBlocks}, g.options().dtype(at::kDouble));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  sqnorm_stage1<<<kNormBlocks, kNormThreads, 0, st>>>(g.data_ptr<float>(), g.numel(), part.data_ptr<double>());
  sqnorm_stage2<<<1, kNormThreads, 0, st>>>(part.data_ptr<double>(), kNormBlocks, out.data_ptr<double>(), scale);
  count_launch(2);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void cast_f32_bf16(torch::Tensor x, torch::Tensor y) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && y.scalar_type() == at::kBFloat16 && x.numel() == y.numel() &&
                  x.is_contiguous() && y.is_contiguous(),
              "cast_f32_bf16");
  c10::cuda::CUDAGuard guard(x.device());
  const long n = x.numel();
  if (!n) return;
  cast_f32_bf16_kernel<<<grid_for(n, 1), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), reinterpret_cast<bf16*>(y.data_ptr()), n);
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void scale_f32(torch::Tensor x, double s) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous(), "scale_f32");
  c10::cuda::CUDAGuard guard(x.device());
  const long n = x.numel();
  if (!n) return;
  scale_f32_kernel<<<grid_for(n, 1), 256, 0, at::cuda::getCurrentCUDAStream()>>>(x.data_ptr<float>(), n, (float)s);
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

DTB_DEFINE_STATUS_READER(status_optim)

}  // namespace dtb
