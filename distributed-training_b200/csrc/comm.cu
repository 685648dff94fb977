// NVLink / NVSwitch collectives over peer-mapped ("symmetric") device buffers.
//
// Replaces the reference's TCP collectives (dtrain/comm.py:292-391): ring and
// direct all-reduce, reduce-scatter, all-gather, broadcast, barrier.  One process
// per GPU; every rank allocates its buffers with cudaMalloc, exports them with
// cudaIpcGetMemHandle and maps its peers' buffers (the handles travel through the
// rendezvous store).  Kernels then read and write peer memory directly with
// ordinary loads and stores over NVLink - no TMA.  The optional NVLS methods
// (allreduce_nvls, reduce_scatter_nvls) use multimem instructions on an NVSwitch
// multicast mapping instead (see the NVLS section).
//
// Summation orders are fixed so results are bit-identical on every rank:
//   ORDER_RANK   : x_0 + x_1 + ... + x_{W-1}        (dtrain "direct", comm.py:374-391)
//   ORDER_CYCLIC : chunk c summed x_c + x_{c+1} + ... + x_{c-1}  (dtrain "ring",
//                  comm.py:342-355: the chunk travels round the ring from rank c)
// In a two-shot all-reduce the owner of each chunk reduces it in that order and
// everyone copies the owner's result, so all ranks hold identical bits.
//
// Synchronisation: per-CTA flags.  CTA b of rank r writes an epoch number into
// slot [b][r] of every peer's signal pad (release, system scope) and waits until
// slot [b][p] of its own pad reaches the epoch for every peer p (acquire).  The
// same CTA index handles the same slice of every chunk on every rank, so CTA-level
// barriers are enough.  Each wait gives up after `timeout_ns` (%globaltimer),
// writes kStatusPeerTimeout into a host-mapped status word and makes the kernel
// return: a dead peer produces an error on the host, not a hung GPU.
//
// Epochs live on the device: a counter in each rank's own signal pad holds the
// last epoch its collectives used; a kernel reads it once at entry and its last
// CTA to finish advances it.  Nothing about a collective's launch therefore
// changes from call to call, so collectives can be captured in a CUDA graph
// (e.g. the DDP bucket all-reduces inside the captured backward) and replayed.
//
// Lean variants (128 threads, <= 56 registers, < 768 B of static shared memory)
// run beside the GEMM and attention kernels: those are capped at 144 / 152
// registers a thread (common.cuh) and use up to ~226 KB of shared memory per SM,
// which leaves room for exactly such a CTA, so a bucket all-reduce launched during
// backward does not wait for (or take) whole SMs.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <map>
#include <mutex>

#include "comm_engine.h"
#include "common.cuh"

namespace dtb {

constexpr int kMaxRanks = 8;
constexpr int kMaxCommBlocks = 160;
constexpr int kCommThreads = 512;
constexpr int kLeanThreads = 128;

int64_t allreduce(std::vector<int64_t> sigs, int64_t rank, std::vector<int64_t> bufs, int64_t byte_offset, int64_t n,
                  int64_t in_dtype, int64_t out_ptr, int64_t out_dtype, int64_t algo, int64_t order, double scale,
                  double timeout_s, int64_t blocks, bool lean, std::vector<int64_t> sq_pads, int64_t sq_base,
                  int64_t sq_stride);
int64_t reduce_scatter(std::vector<int64_t> sigs, int64_t rank, std::vector<int64_t> bufs,
                       int64_t byte_offset, int64_t n, int64_t dtype, int64_t out_ptr, int64_t order, double scale,
                       int64_t sq_part_ptr, double timeout_s, int64_t blocks);
int64_t all_gather(std::vector<int64_t> sigs, int64_t rank, std::vector<int64_t> bufs,
                   int64_t byte_offset, int64_t n, int64_t dtype, double timeout_s, int64_t blocks);
int64_t device_barrier(std::vector<int64_t> sigs, int64_t rank, double timeout_s);
int64_t allreduce_nvls(std::vector<int64_t> sigs, int64_t rank, int64_t mc_ptr, int64_t byte_offset, int64_t n,
                       int64_t dtype, double scale, double timeout_s, int64_t blocks, bool lean,
                       std::vector<int64_t> sq_pads, int64_t sq_base, int64_t sq_stride);
int64_t reduce_scatter_nvls(std::vector<int64_t> sigs, int64_t rank, int64_t mc_ptr, int64_t byte_offset, int64_t n,
                            int64_t out_ptr, double scale, int64_t sq_part_ptr, double timeout_s, int64_t blocks);

enum : int { ORDER_RANK = 0, ORDER_CYCLIC = 1 };
enum : int { DT_F32 = 0, DT_BF16 = 1 };

struct Peers {
  void* p[kMaxRanks];
};
struct Sigs {
  uint32_t* p[kMaxRanks];
};

struct CommCtx {
  Sigs sig;           // every rank's signal pad [kMaxCommBlocks][kMaxRanks] + descriptor ring + counters
  const Sigs* sp;     // device: a shared-memory copy of `sig` (set by collective_begin)
  int rank, world;
  uint32_t epoch;     // first epoch of this launch: set on the device by collective_begin()
  uint32_t tag;       // descriptor of this collective (kind, element count, dtype)
  uint64_t timeout_ns;
  int* host_status;   // host-mapped status word (device pointer)
};

// Sums of squares of a collective's reduced values, published to every rank:
// CTA b of rank r writes its slice's fp64 sum to p[q][r * stride + base + b] on
// every rank q, so each rank ends up with all ranks' partials in its own pad.
struct SqOut {
  double* p[kMaxRanks];  // every rank's pad (nullptr: not requested)
  int base, stride;
};

// After the flags, each rank's signal pad holds a ring of kDescSlots 64-bit
// descriptors (epoch << 32 | tag) of its own recent collectives, then three 32-bit
// words: the last epoch used, the CTAs of the running collective that exited, and
// a "failed" flag that a timed-out wait sets (device memory, so every later wait
// can check it cheaply and give up at once instead of waiting out its own timeout).
constexpr int kFlagWords = kMaxCommBlocks * kMaxRanks;
constexpr int kDescSlots = 16;
constexpr int kCtrWord = kFlagWords + 2 * kDescSlots;
constexpr int kFailWord = kCtrWord + 2;
constexpr int kSigBytesUsed = (kCtrWord + 3) * 4;
static_assert(kSigBytesUsed <= 8192, "signal pad layout exceeds the 8 KB pad");

// Copies pointer arrays from kernel parameters into shared memory with static
// indices.  The kernels index them with ranks computed at run time; doing that on
// the parameters would make every thread keep a local-memory copy of the struct.
#define DTB_SHARED_COPY(T, name, src)                                      \
  __shared__ T name;                                                      \
  if (threadIdx.x == 0) {                                                 \
    _Pragma("unroll") for (int i_ = 0; i_ < kMaxRanks; ++i_) name.p[i_] = (src).p[i_]; \
  }

// Reads the epoch counter (one value for the whole CTA): this launch uses epochs
// last+1 ... last+used.  Also publishes the shared copies the kernel made before
// calling it (its barriers order them).
__device__ __forceinline__ void collective_begin(CommCtx& c) {
  DTB_SHARED_COPY(Sigs, s_sig, c.sig)
  __shared__ uint32_t s_last;
  __syncthreads();
  if (threadIdx.x == 0) s_last = __ldcg(s_sig.p[c.rank] + kCtrWord);  // L2: written by the last launch
  __syncthreads();
  c.sp = &s_sig;
  c.epoch = s_last + 1u;
}

// Every CTA calls this once on its way out (also after a timeout); the last one
// resets the exit count and advances the epoch counter by `used`.  All CTAs have
// read the counter before any of them can be the last to exit.
__device__ __forceinline__ void collective_end(const CommCtx& c, uint32_t used) {
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* w = c.sp->p[c.rank] + kCtrWord;
    __threadfence();
    if (atomicAdd(w + 1, 1u) == gridDim.x - 1u) {
      atomicExch(w + 1, 0u);
      atomicExch(w, c.epoch - 1u + used);
      __threadfence();
    }
  }
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Polling load: relaxed at system scope, so it reads the coherent value without
// the L1 invalidation an acquire implies on every poll (a co-resident kernel keeps
// its L1 contents); the waiter issues one acquire fence once the flag has arrived.
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acquire_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ uint64_t ld_acquire_sys64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool group_failed(const CommCtx& c) {
  return *reinterpret_cast<volatile const uint32_t*>(c.sp->p[c.rank] + kFailWord) != 0u;
}
__device__ __forceinline__ void mark_failed(const CommCtx& c) {
  atomicExch(c.sp->p[c.rank] + kFailWord, 1u);
  atomicCAS(c.host_status, 0, kStatusPeerTimeout);
  set_status(kStatusPeerTimeout);
}

// CTA-level barrier across ranks.  Returns false if a peer did not arrive in time.
__device__ bool cta_barrier(const CommCtx& c, uint32_t epoch) {
  __shared__ int failed;
  __syncthreads();
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if (threadIdx.x < c.world) {
    const int p = threadIdx.x;
    __threadfence_system();
    st_release_sys(c.sp->p[p] + blockIdx.x * kMaxRanks + c.rank, epoch);
    const uint32_t* mine = c.sp->p[c.rank] + blockIdx.x * kMaxRanks + p;
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
      const uint32_t v = ld_relaxed_sys(mine);
      if ((int)(v - epoch) >= 0) {
        fence_acquire_sys();
        break;
      }
      // after a short spin, poll politely: the CTA may share its SM with a GEMM
      if (i >= 16u) __nanosleep(i < 256u ? 128 : 512);
      if ((i & 31u) == 0u) {
        const uint64_t now = globaltimer_ns();
        if (t0 == 0) t0 = now;
        // a collective of this group already failed (a peer is gone): give up now
        // rather than wait out another full timeout in every queued collective
        if (group_failed(c) || (t0 != now && now - t0 > c.timeout_ns)) {
          atomicExch(&failed, 1);
          mark_failed(c);
          break;
        }
      }
    }
  }
  __syncthreads();
  return failed == 0;
}

// First barrier of a collective, with desynchronisation detection: CTA 0 publishes
// this rank's descriptor of the collective for its epoch before arriving and, once
// every peer has arrived at the epoch, compares the peers' descriptors for the same
// epoch with its own.  Ranks that issued different collectives (or sizes) at the
// same point get kStatusSeqMismatch and return instead of mixing unrelated data.
// (A peer cannot overwrite that slot before this rank reaches the collective's next
// barrier, so the ring never aliases.)
__device__ bool cta_enter(const CommCtx& c) {
  const uint64_t mine = ((uint64_t)c.epoch << 32) | c.tag;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    uint64_t* ring = reinterpret_cast<uint64_t*>(c.sp->p[c.rank] + kFlagWords);
    *reinterpret_cast<volatile uint64_t*>(ring + (c.epoch % kDescSlots)) = mine;
    __threadfence_system();
  }
  if (!cta_barrier(c, c.epoch)) return false;
  if (blockIdx.x != 0) return true;
  __shared__ int mismatch;
  if (threadIdx.x == 0) mismatch = 0;
  __syncthreads();
  if (threadIdx.x < c.world && threadIdx.x != c.rank) {
    const uint64_t* ring = reinterpret_cast<const uint64_t*>(c.sp->p[threadIdx.x] + kFlagWords);
    if (ld_acquire_sys64(ring + (c.epoch % kDescSlots)) != mine) {
      atomicExch(&mismatch, 1);
      atomicCAS(c.host_status, 0, kStatusSeqMismatch);
      atomicExch(c.sp->p[c.rank] + kFailWord, 1u);
      set_status(kStatusSeqMismatch);
    }
  }
  __syncthreads();
  return mismatch == 0;
}

// [lo, hi) of chunk `c` of an n-element buffer split over W ranks: the first
// n % W chunks get one extra element (dtrain/comm.py:220-226).
__device__ __forceinline__ void chunk_bounds(long n, int W, int c, long& lo, long& hi) {
  const long base = n / W, extra = n % W;
  lo = c * base + min((long)c, extra);
  hi = lo + base + (c < extra ? 1 : 0);
}

// Sub-range of [lo, hi) handled by this CTA (same on every rank).
__device__ __forceinline__ void cta_slice(long lo, long hi, long& a, long& b) {
  const long len = hi - lo;
  const long per = (((len + gridDim.x - 1) / gridDim.x) + 63) & ~63L;
  a = min(hi, lo + (long)blockIdx.x * per);
  b = min(hi, a + per);
}

template <typename T>
__device__ __forceinline__ float ldf(const T* p);
template <>
__device__ __forceinline__ float ldf<float>(const float* p) { return __ldcg(p); }
template <>
__device__ __forceinline__ float ldf<bf16>(const bf16* p) {
  unsigned short u = __ldcg(reinterpret_cast<const unsigned short*>(p));
  return __uint_as_float(((uint32_t)u) << 16);
}
template <typename T>
__device__ __forceinline__ void stf(T* p, float v);
template <>
__device__ __forceinline__ void stf<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void stf<bf16>(bf16* p, float v) { *p = f2bf(v); }

// Reduce x[i] over ranks in the given order (starting rank `first`).
template <typename TI>
__device__ __forceinline__ float reduce_elem(const Peers& in, long i, int W, int first) {
  int r = first;
  float acc = ldf(reinterpret_cast<const TI*>(in.p[r]) + i);
  for (int k = 1; k < W; ++k) {
    r = (r + 1 == W) ? 0 : r + 1;
    acc += ldf(reinterpret_cast<const TI*>(in.p[r]) + i);
  }
  return acc;
}

// Vectorised fp32 reduction of 4 elements starting at i.  With a compile-time
// world size (WT > 0) every peer's load is issued before the first add, so a
// thread keeps WT 16-byte loads in flight over NVLink (the loop is latency
// bound otherwise); the adds still run in the fixed order first, first+1, ...
template <int WT>
__device__ __forceinline__ float4 reduce_vec4(const Peers& in, long i, int W, int first) {
  if constexpr (WT > 0) {
    float4 v[WT];
#pragma unroll
    for (int k = 0; k < WT; ++k) {
      int r = first + k;
      r -= (r >= WT) ? WT : 0;
      v[k] = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(in.p[r]) + i));
    }
    float4 acc = v[0];
#pragma unroll
    for (int k = 1; k < WT; ++k) {
      acc.x += v[k].x; acc.y += v[k].y; acc.z += v[k].z; acc.w += v[k].w;
    }
    return acc;
  } else {
    int r = first;
    float4 acc = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(in.p[r]) + i));
    for (int k = 1; k < W; ++k) {
      r = (r + 1 == W) ? 0 : r + 1;
      const float4 v = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(in.p[r]) + i));
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    return acc;
  }
}

// Vectorised bf16 reduction of 8 elements starting at i (one 16-byte load per
// rank, all issued before the first add), summed in fp32 in the fixed order
// first, first+1, ... exactly like reduce_elem<bf16>.
template <int WT>
__device__ __forceinline__ void reduce_vec8_bf16(const Peers& in, long i, int W, int first, float* acc) {
  auto add8 = [&](const uint4& u, bool init) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      acc[2 * e] = init ? f.x : acc[2 * e] + f.x;
      acc[2 * e + 1] = init ? f.y : acc[2 * e + 1] + f.y;
    }
  };
  if constexpr (WT > 0) {
    uint4 v[WT];
#pragma unroll
    for (int k = 0; k < WT; ++k) {
      int r = first + k;
      r -= (r >= WT) ? WT : 0;
      v[k] = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(in.p[r]) + i));
    }
#pragma unroll
    for (int k = 0; k < WT; ++k) add8(v[k], k == 0);
  } else {
    int r = first;
    for (int k = 0; k < W; ++k) {
      add8(__ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(in.p[r]) + i)), k == 0);
      r = (r + 1 == W) ? 0 : r + 1;
    }
  }
}

template <typename TO>
__device__ __forceinline__ void store8(TO* out, const float* v);
template <>
__device__ __forceinline__ void store8<float>(float* out, const float* v) {
  *reinterpret_cast<float4*>(out) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(out + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
template <>
__device__ __forceinline__ void store8<bf16>(bf16* out, const float* v) {
  *reinterpret_cast<uint4*>(out) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                              pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}

// Reduce elements [a, b) into `out` (index space of the buffer), scaled.
// If sq != nullptr, also accumulate sum of squares of the written values (fp64).
// All ranks' buffers share one byte offset from 256-byte aligned bases, so they
// have the same 16-byte phase; the vector loop runs when `out` shares it too.
template <typename TI, typename TO, int WT = 0, bool LEAN = false>
__device__ __forceinline__ void reduce_range(const Peers& in, TO* out, long a, long b, int W, int first, float scale,
                                             double* sq) {
  double s = 0.0;
  if (a >= b) { if (sq) *sq += s; return; }
  if constexpr (std::is_same<TI, float>::value && std::is_same<TO, float>::value) {
    const uintptr_t ain = reinterpret_cast<uintptr_t>(reinterpret_cast<const float*>(in.p[first]) + a);
    const uintptr_t aout = reinterpret_cast<uintptr_t>(out + a);
    long head = a, ve = a;
    if (((ain ^ aout) & 15) == 0 && (ain & 3) == 0) {
      head = min(b, a + (long)(((16 - (ain & 15)) & 15) / 4));
      ve = head + ((b - head) & ~3L);
    }
    for (long i = a + threadIdx.x; i < head; i += blockDim.x) {
      const float v = reduce_elem<TI>(in, i, W, first) * scale;
      out[i] = v;
      s += (double)v * v;
    }
    // two float4 per thread per iteration: 2*WT loads in flight (one in the lean
    // variant, which has a quarter of the registers)
    const long step = (long)blockDim.x * 4;
    long i = head + threadIdx.x * 4;
    for (; !LEAN && i + step < ve; i += 2 * step) {
      float4 v0 = reduce_vec4<WT>(in, i, W, first);
      float4 v1 = reduce_vec4<WT>(in, i + step, W, first);
      v0.x *= scale; v0.y *= scale; v0.z *= scale; v0.w *= scale;
      v1.x *= scale; v1.y *= scale; v1.z *= scale; v1.w *= scale;
      *reinterpret_cast<float4*>(out + i) = v0;
      *reinterpret_cast<float4*>(out + i + step) = v1;
      if (sq) {
        s += (double)v0.x * v0.x + (double)v0.y * v0.y + (double)v0.z * v0.z + (double)v0.w * v0.w;
        s += (double)v1.x * v1.x + (double)v1.y * v1.y + (double)v1.z * v1.z + (double)v1.w * v1.w;
      }
    }
    for (; i < ve; i += step) {
      float4 v = reduce_vec4<WT>(in, i, W, first);
      v.x *= scale; v.y *= scale; v.z *= scale; v.w *= scale;
      *reinterpret_cast<float4*>(out + i) = v;
      if (sq) s += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
    }
    for (long i = max(ve, head) + threadIdx.x; i < b; i += blockDim.x) {
      const float v = reduce_elem<TI>(in, i, W, first) * scale;
      out[i] = v;
      s += (double)v * v;
    }
  } else if constexpr (std::is_same<TI, bf16>::value) {
    // 8 bf16 per vector: input phase 16 B, output phase 16 B (bf16) or 32 B (fp32)
    const uintptr_t ain = reinterpret_cast<uintptr_t>(reinterpret_cast<const bf16*>(in.p[first]) + a);
    const uintptr_t aout = reinterpret_cast<uintptr_t>(out + a);
    constexpr uintptr_t kOutAlign = 16;
    long head = a, ve = a;
    if ((ain & 1) == 0) {
      const long to_in = (long)(((16 - (ain & 15)) & 15) / 2);
      const uintptr_t out_at = aout + to_in * sizeof(TO);
      if ((out_at & (kOutAlign - 1)) == 0) {
        head = min(b, a + to_in);
        ve = head + ((b - head) & ~7L);
      }
    }
    for (long i = a + threadIdx.x; i < head; i += blockDim.x) {
      const float v = reduce_elem<TI>(in, i, W, first) * scale;
      stf<TO>(out + i, v);
      s += (double)v * v;
    }
    // two vectors per thread per iteration: 2*WT 16-byte loads in flight (one
    // vector in the lean variant)
    const long step = (long)blockDim.x * 8;
    long i = head + threadIdx.x * 8;
    for (; !LEAN && i + step < ve; i += 2 * step) {
      float v0[8], v1[8];
      reduce_vec8_bf16<WT>(in, i, W, first, v0);
      reduce_vec8_bf16<WT>(in, i + step, W, first, v1);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v0[e] *= scale;
        v1[e] *= scale;
        if (sq) s += (double)v0[e] * v0[e] + (double)v1[e] * v1[e];
      }
      store8<TO>(out + i, v0);
      store8<TO>(out + i + step, v1);
    }
    for (; i < ve; i += step) {
      float v[8];
      reduce_vec8_bf16<WT>(in, i, W, first, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[e] *= scale;
        if (sq) s += (double)v[e] * v[e];
      }
      store8<TO>(out + i, v);
    }
    for (long i = max(ve, head) + threadIdx.x; i < b; i += blockDim.x) {
      const float v = reduce_elem<TI>(in, i, W, first) * scale;
      stf<TO>(out + i, v);
      s += (double)v * v;
    }
  } else {
    for (long i = a + threadIdx.x; i < b; i += blockDim.x) {
      const float v = reduce_elem<TI>(in, i, W, first) * scale;
      stf<TO>(out + i, v);
      s += (double)v * v;
    }
  }
  if (sq) *sq += s;
}

// Copy elements [a, b) from src to dst (typically peer -> local) with 16-byte
// vectors when both pointers share a 16-byte phase.
template <typename T>
__device__ __forceinline__ void copy_range(const T* src, T* dst, long a, long b) {
  const char* s = reinterpret_cast<const char*>(src + a);
  char* d = reinterpret_cast<char*>(dst + a);
  const long nbytes = (b - a) * (long)sizeof(T);
  if (nbytes <= 0) return;
  const uintptr_t ps = reinterpret_cast<uintptr_t>(s), pd = reinterpret_cast<uintptr_t>(d);
  if (((ps ^ pd) & 15) == 0) {
    const long head = min(nbytes, (long)((16 - (ps & 15)) & 15));
    const long nv = (nbytes - head) / 16;
    for (long i = threadIdx.x; i < head; i += blockDim.x) d[i] = s[i];
    const uint4* sv = reinterpret_cast<const uint4*>(s + head);
    uint4* dv = reinterpret_cast<uint4*>(d + head);
    // four independent 16-byte loads per thread in flight
    const long st = blockDim.x;
    long i = threadIdx.x;
    for (; i + 3 * st < nv; i += 4 * st) {
      const uint4 x0 = __ldcg(sv + i), x1 = __ldcg(sv + i + st), x2 = __ldcg(sv + i + 2 * st),
                  x3 = __ldcg(sv + i + 3 * st);
      dv[i] = x0;
      dv[i + st] = x1;
      dv[i + 2 * st] = x2;
      dv[i + 3 * st] = x3;
    }
    for (; i < nv; i += st) dv[i] = __ldcg(sv + i);
    for (long i = head + nv * 16 + threadIdx.x; i < nbytes; i += blockDim.x) d[i] = s[i];
  } else {
    for (long i = threadIdx.x; i < nbytes; i += blockDim.x) d[i] = s[i];
  }
}

// ---------------------------------------------------------------- kernels
// One-shot all-reduce: every rank reduces the whole buffer from all peers (order
// ORDER_RANK or ORDER_CYCLIC over the same chunking as the two-shot) into `out`.
template <typename TI, typename TO, int WT>
__device__ __forceinline__ void allreduce_oneshot_body(CommCtx c, const Peers& in, TO* out, long n, int order, float scale) {
  if (!cta_enter(c)) return;
  for (int ch = 0; ch < c.world; ++ch) {
    long lo, hi, a, b;
    chunk_bounds(n, c.world, ch, lo, hi);
    cta_slice(lo, hi, a, b);
    reduce_range<TI, TO, WT>(in, out, a, b, c.world, order == ORDER_CYCLIC ? ch : 0, scale, nullptr);
  }
  cta_barrier(c, c.epoch + 1);
}
template <typename TI, typename TO, int WT>
__global__ void __launch_bounds__(kCommThreads)
    allreduce_oneshot_kernel(CommCtx c, Peers in, TO* out, long n, int order, float scale) {
  DTB_SHARED_COPY(Peers, s_in, in)
  collective_begin(c);
  allreduce_oneshot_body<TI, TO, WT>(c, s_in, out, n, order, scale);
  collective_end(c, 2);
}

// Fixed-order block sum of a per-thread fp64 value; thread q < W then stores it
// into rank q's pad at [rank * stride + base + blockIdx.x].  The cta_barrier that
// follows has the same thread q release its flag to rank q, which orders the store
// before the peer passes that barrier.
template <int NT>
__device__ __forceinline__ void publish_sq(const CommCtx& c, const SqOut& sq, double s) {
  __shared__ double red[NT / 32];
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < c.world) {
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) t += red[w];
    sq.p[threadIdx.x][(long)c.rank * sq.stride + sq.base + blockIdx.x] = t;
  }
}

// Two-shot all-reduce: reduce-scatter into the owner's buffer (in place), then
// all-gather of the reduced chunks.  `out` is this rank's destination (may be the
// local input buffer).  in.p[rank] must be this rank's input; in-place is safe
// because the owner only writes its own chunk, which peers do not read until the
// middle barrier.  With `sq` the owner also publishes the sum of squares of the
// scaled values it reduced (the DDP gradient norm comes out of the all-reduce, not
// out of a second pass over the gradient).  LEAN: 128-thread CTAs that fit beside
// a GEMM or attention CTA on one SM (used for buckets reduced during backward).
template <typename T, int WT, bool LEAN>
__device__ __forceinline__ void allreduce_twoshot_body(CommCtx c, const Peers& in, T* out, long n, int order, float scale,
                                                       const SqOut& sq) {
  if (!cta_enter(c)) return;
  long lo, hi, a, b;
  chunk_bounds(n, c.world, c.rank, lo, hi);
  cta_slice(lo, hi, a, b);
  T* mine = reinterpret_cast<T*>(in.p[c.rank]);
  const bool want_sq = sq.p[0] != nullptr;
  double s = 0.0;
  reduce_range<T, T, WT, LEAN>(in, mine, a, b, c.world, order == ORDER_CYCLIC ? c.rank : 0, scale,
                               want_sq ? &s : nullptr);
  if (want_sq) publish_sq<LEAN ? kLeanThreads : kCommThreads>(c, sq, s);
  if (!cta_barrier(c, c.epoch + 1)) return;
  for (int k = 0; k < c.world; ++k) {
    const int p = (c.rank + k) % c.world;
    chunk_bounds(n, c.world, p, lo, hi);
    cta_slice(lo, hi, a, b);
    if (p == c.rank) {
      if (out != mine) copy_range<T>(mine, out, a, b);
    } else {
      copy_range<T>(reinterpret_cast<const T*>(in.p[p]), out, a, b);
    }
  }
  cta_barrier(c, c.epoch + 2);
}
template <typename T, int WT, bool LEAN>
__global__ void __maxnreg__(LEAN ? DTB_LEAN_COMM_MAXNREG : 128)
    allreduce_twoshot_kernel(CommCtx c, Peers in, T* out, long n, int order, float scale, SqOut sq) {
  DTB_SHARED_COPY(Peers, s_in, in)
  DTB_SHARED_COPY(SqOut, s_sq, sq)
  if (threadIdx.x == 0) {
    s_sq.base = sq.base;
    s_sq.stride = sq.stride;
  }
  collective_begin(c);
  allreduce_twoshot_body<T, WT, LEAN>(c, s_in, out, n, order, scale, s_sq);
  collective_end(c, 3);
}

// ---------------------------------------------------------------- NVLS
// Switch-side reduction through an NVSwitch multicast mapping (one address that
// covers the same offset of every rank's buffer, see vmm.cpp):
//   multimem.ld_reduce  returns the sum over all ranks of the values at that offset,
//                       added in the switch (fp32; bf16 pairs with fp32 accumulation);
//   multimem.st         writes a value to that offset of every rank's buffer.
// All-reduce: each rank reduces its share of the buffer with ld_reduce and stores
// the (scaled) sums back through the multicast address, so every element is summed
// once and every rank receives the same bits.  Per GPU that moves about
// (1 + 1/W) x size each way over NVLink, against 2 (W-1)/W x size for the two-shot
// kernel: less from W = 4 up.  The order of the switch's additions is the
// hardware's, not the ring or rank order, so this path is an opt-in method
// (ranks still agree bit for bit).  Reduce-scatter: each rank reduces its own
// partition with ld_reduce and stores it locally; only 1/W of the data enters
// each GPU.
__device__ __forceinline__ float4 mm_ld_add_v4f32(const void* p) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ float mm_ld_add_f32(const void* p) {
  float v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint4 mm_ld_add_v4bf16x2(const void* p) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void mm_st_v4f32(void* p, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void mm_st_v4bf16x2(void* p, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void mm_st_f32(void* p, float v) {
  asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

constexpr int kNvlsUnroll = 4;  // independent switch reductions in flight per thread

// Scale one reduced 16-byte vector and add its squares to `s` (fp64).
__device__ __forceinline__ float4 nvls_scale(float4 v, float scale, bool want_sq, double& s) {
  v.x *= scale; v.y *= scale; v.z *= scale; v.w *= scale;
  if (want_sq) s += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
  return v;
}
__device__ __forceinline__ uint4 nvls_scale(uint4 v, float scale, bool want_sq, double& s) {
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float lo = __uint_as_float(w[e] << 16) * scale, hi = __uint_as_float(w[e] & 0xffff0000u) * scale;
    if (want_sq) s += (double)lo * lo + (double)hi * hi;
    w[e] = pack_bf16x2(lo, hi);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// All-reduce through the switch.  The buffer is split into 16-byte vectors; rank r
// owns vectors chunk_bounds(nvec, W, r), and rank 0 also owns the fp32 elements
// before the first and after the last whole vector (a buffer that does not start on
// a 16-byte boundary; bf16 buffers must, and hold whole vectors).  `mc` is the
// multicast address of the data.  With `sq` each CTA publishes the sum of squares
// of the values it stored, as the two-shot kernel does.  LEAN: 128-thread CTAs that
// fit beside a GEMM or attention CTA (buckets reduced during backward).
template <typename T, bool LEAN>
__global__ void __maxnreg__(LEAN ? DTB_LEAN_COMM_MAXNREG : 128)
    allreduce_nvls_kernel(CommCtx c, char* mc, long n, float scale, SqOut sq) {
  using V = typename std::conditional<std::is_same<T, float>::value, float4, uint4>::type;
  constexpr int kPerVec = 16 / (int)sizeof(T);
  DTB_SHARED_COPY(SqOut, s_sq, sq)
  if (threadIdx.x == 0) {
    s_sq.base = sq.base;
    s_sq.stride = sq.stride;
  }
  collective_begin(c);
  if (cta_enter(c)) {
    const bool want_sq = s_sq.p[0] != nullptr;
    // elements before the first 16-byte boundary (fp32 only), then whole vectors
    const long head = min(n, (long)((16 - (reinterpret_cast<uintptr_t>(mc) & 15)) & 15) / (long)sizeof(T));
    char* mv = mc + head * (long)sizeof(T);
    const long nvec = (n - head) / kPerVec;
    long lo, hi, a, b;
    chunk_bounds(nvec, c.world, c.rank, lo, hi);
    cta_slice(lo, hi, a, b);
    double s = 0.0;
    const long stride = (long)blockDim.x;
    for (long v0 = a + threadIdx.x; v0 < b; v0 += kNvlsUnroll * stride) {
      V x[kNvlsUnroll];
#pragma unroll
      for (int u = 0; u < kNvlsUnroll; ++u) {
        const long v = v0 + u * stride;
        if (v < b) {
          if constexpr (std::is_same<T, float>::value) x[u] = mm_ld_add_v4f32(mv + v * 16);
          else x[u] = mm_ld_add_v4bf16x2(mv + v * 16);
        }
      }
#pragma unroll
      for (int u = 0; u < kNvlsUnroll; ++u) {
        const long v = v0 + u * stride;
        if (v < b) {
          const V y = nvls_scale(x[u], scale, want_sq, s);
          if constexpr (std::is_same<T, float>::value) mm_st_v4f32(mv + v * 16, y);
          else mm_st_v4bf16x2(mv + v * 16, y);
        }
      }
    }
    if constexpr (std::is_same<T, float>::value) {
      if (c.rank == 0 && blockIdx.x == 0) {
        const long tail = head + nvec * kPerVec;
        for (long i = threadIdx.x; i < head + (n - tail); i += stride) {
          const long e = i < head ? i : tail + (i - head);
          const float y = mm_ld_add_f32(mc + e * 4) * scale;
          if (want_sq) s += (double)y * y;
          mm_st_f32(mc + e * 4, y);
        }
      }
    }
    if (want_sq) publish_sq<LEAN ? kLeanThreads : kCommThreads>(c, s_sq, s);
    cta_barrier(c, c.epoch + 1);
  }
  collective_end(c, 2);
}

// Reduce-scatter (fp32) through the switch: this rank's partition
// chunk_bounds(n, W, rank) of the buffer is summed over ranks by ld_reduce, scaled
// and stored into `out` (this rank's buffer, same index space).  The partition's
// unaligned head and tail elements go through scalar reductions.  With sq_part,
// CTA b writes the fp64 sum of squares of its slice to sq_part[b].
__global__ void __launch_bounds__(kCommThreads)
    reduce_scatter_nvls_kernel(CommCtx c, const char* mc, float* out, long n, float scale, double* sq_part) {
  __shared__ double red[kCommThreads / 32];
  collective_begin(c);
  if (cta_enter(c)) {
    long lo, hi;
    chunk_bounds(n, c.world, c.rank, lo, hi);
    const long vlo = (lo + 3) / 4, vhi = hi / 4;  // whole 16-byte vectors inside [lo, hi)
    double s = 0.0;
    const long stride = (long)blockDim.x;
    if (vlo < vhi) {
      long a, b;
      cta_slice(vlo, vhi, a, b);
      for (long v0 = a + threadIdx.x; v0 < b; v0 += kNvlsUnroll * stride) {
        float4 x[kNvlsUnroll];
#pragma unroll
        for (int u = 0; u < kNvlsUnroll; ++u) {
          const long v = v0 + u * stride;
          if (v < b) x[u] = mm_ld_add_v4f32(mc + v * 16);
        }
#pragma unroll
        for (int u = 0; u < kNvlsUnroll; ++u) {
          const long v = v0 + u * stride;
          if (v < b) *reinterpret_cast<float4*>(out + v * 4) = nvls_scale(x[u], scale, sq_part != nullptr, s);
        }
      }
    }
    if (blockIdx.x == 0) {
      // elements of [lo, hi) outside the whole vectors (all of them if there are none)
      const long h_end = vlo < vhi ? vlo * 4 : hi, t_beg = vlo < vhi ? vhi * 4 : hi;
      for (long i = lo + threadIdx.x; i < h_end; i += stride) {
        const float y = mm_ld_add_f32(mc + i * 4) * scale;
        s += (double)y * y;
        out[i] = y;
      }
      for (long i = t_beg + threadIdx.x; i < hi; i += stride) {
        const float y = mm_ld_add_f32(mc + i * 4) * scale;
        s += (double)y * y;
        out[i] = y;
      }
    }
    if (sq_part) {
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
      __syncthreads();
      if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
        sq_part[blockIdx.x] = t;
      }
    }
    cta_barrier(c, c.epoch + 1);
  }
  collective_end(c, 2);
}

// Sum of fp64 partials pad[r * stride + s] over ranks r < world and slots
// lo <= s < hi, in a fixed order (thread t sums the linear indices t, t+1024, ...
// of that range in order, then a fixed shuffle tree): the same bits on every rank.
__global__ void __launch_bounds__(1024)
    sq_total_kernel(const double* pad, int world, long stride, long lo, long hi, double* out) {
  __shared__ double red[32];
  const long len = hi - lo, n = (long)world * len;
  double s = 0.0;
  for (long i = threadIdx.x; i < n; i += blockDim.x) s += __ldcg(pad + (i / len) * stride + lo + i % len);
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < 32; ++w) t += red[w];
    out[0] = t;
  }
}

// Reduce-scatter: chunk `rank` summed in cyclic order from `rank` (bit-equal to
// dtrain's ring reduce-scatter with rotation, comm.py:310-316,342-362), scaled,
// written to `out` (this rank's buffer index space).  With sq_part, each CTA also
// writes the fp64 sum of squares of its slice to sq_part[blockIdx.x].
template <typename TI, typename TO, int WT>
__device__ __forceinline__ void reduce_scatter_body(CommCtx c, const Peers& in, TO* out, long n, int order, float scale, double* sq_part) {
  __shared__ double red[kCommThreads / 32];
  if (!cta_enter(c)) return;
  long lo, hi, a, b;
  chunk_bounds(n, c.world, c.rank, lo, hi);
  cta_slice(lo, hi, a, b);
  double s = 0.0;
  reduce_range<TI, TO, WT>(in, out, a, b, c.world, order == ORDER_CYCLIC ? c.rank : 0, scale,
                           sq_part ? &s : nullptr);
  if (sq_part) {
    // fixed-order block reduction
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = 0.0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
      sq_part[blockIdx.x] = t;
    }
  }
  cta_barrier(c, c.epoch + 1);
}
template <typename TI, typename TO, int WT>
__global__ void __launch_bounds__(kCommThreads)
    reduce_scatter_kernel(CommCtx c, Peers in, TO* out, long n, int order, float scale, double* sq_part) {
  DTB_SHARED_COPY(Peers, s_in, in)
  collective_begin(c);
  reduce_scatter_body<TI, TO, WT>(c, s_in, out, n, order, scale, sq_part);
  collective_end(c, 2);
}

// All-gather in place: every rank copies chunk p from rank p into `out`.
template <typename T>
__device__ __forceinline__ void all_gather_body(CommCtx c, const Peers& in, T* out, long n) {
  if (!cta_enter(c)) return;
  for (int k = 1; k < c.world; ++k) {
    const int p = (c.rank + k) % c.world;
    long lo, hi, a, b;
    chunk_bounds(n, c.world, p, lo, hi);
    cta_slice(lo, hi, a, b);
    copy_range<T>(reinterpret_cast<const T*>(in.p[p]), out, a, b);
  }
  cta_barrier(c, c.epoch + 1);
}
template <typename T>
__global__ void __launch_bounds__(kCommThreads)
    all_gather_kernel(CommCtx c, Peers in, T* out, long n) {
  DTB_SHARED_COPY(Peers, s_in, in)
  collective_begin(c);
  all_gather_body<T>(c, s_in, out, n);
  collective_end(c, 2);
}

// Broadcast from `root`: non-root ranks pull root's buffer into `out` (with an
// optional fp32 -> bf16 cast into out16 on every rank, root included).
__device__ __forceinline__ void broadcast_body(CommCtx c, const Peers& in, void* out, long nbytes, int root, const float* cast_src, bf16* out16,
                     long n16) {
  if (!cta_enter(c)) return;
  if (c.rank != root && out) {
    long a, b;
    cta_slice(0, nbytes, a, b);
    copy_range<char>(reinterpret_cast<const char*>(in.p[root]), reinterpret_cast<char*>(out), a, b);
  }
  if (!cta_barrier(c, c.epoch + 1)) return;
  if (out16) {
    long a, b;
    cta_slice(0, n16, a, b);
    for (long i = a + threadIdx.x; i < b; i += blockDim.x) out16[i] = f2bf(cast_src[i]);
  }
}
__global__ void __launch_bounds__(kCommThreads)
    broadcast_kernel(CommCtx c, Peers in, void* out, long nbytes, int root, const float* cast_src, bf16* out16,
                     long n16) {
  DTB_SHARED_COPY(Peers, s_in, in)
  collective_begin(c);
  broadcast_body(c, s_in, out, nbytes, root, cast_src, out16, n16);
  collective_end(c, 2);
}

__global__ void barrier_kernel(CommCtx c) {
  collective_begin(c);
  cta_enter(c);
  collective_end(c, 1);
}

// ZeRO-1 update, fused with the global-norm exchange and the parameter all-gather.
// Phase 1: every CTA sums all ranks' per-CTA squared-norm partials (written by
//          reduce_scatter_kernel into each rank's symmetric sq slot) in rank-then-CTA
//          order -> identical global norm on every rank, then the clip factor.
// Phase 2: AdamW on this rank's shard [lo, hi) of the flat fp32 master (dtrain/zero.py:45-62),
//          writing the fp32 master and the bf16 working copy (symmetric).
// Phase 3: all-gather of the bf16 working copy (and optionally the fp32 master).
//          With `keep` (nkeep sorted [lo, hi) intervals of the flat buffer) only those
//          ranges of the bf16 copy are gathered here: the Linear weights are left to
//          the forward GEMMs that gather them tile by tile (gemm.cu, gemm_gather),
//          which start pulling once `gen_out` (written here) moves past the
//          generation they last gathered.
__device__ __forceinline__ void zero_adamw_allgather_body(CommCtx c, const Sigs& sq_parts, int nparts, float* master, const float* grad,
                                float* m, float* v, const Peers& work16, const Peers& master32, long n, AdamConsts ak,
                                float max_norm, double* sq_out, int gather_master, const long* keep, int nkeep,
                                int* gen_out) {
  __shared__ float s_clip;
  if (!cta_enter(c)) return;
  if (gen_out && blockIdx.x == 0 && threadIdx.x == 0) *gen_out = (int)(c.epoch + 1u);
  if (threadIdx.x == 0) {
    double tot = 0.0;
    for (int r = 0; r < c.world; ++r) {
      const double* pp = reinterpret_cast<const double*>(sq_parts.p[r]);
      double rs = 0.0;
      for (int k = 0; k < nparts; ++k) rs += __ldcg(pp + k);
      tot += rs;
    }
    float cs = 1.f;
    const double nrm = sqrt(tot);
    if (max_norm > 0.f && nrm > (double)max_norm && nrm != 0.0) cs = (float)((double)max_norm / (nrm + 1e-6));
    s_clip = cs;
    if (blockIdx.x == 0 && sq_out) sq_out[0] = tot;
  }
  __syncthreads();
  const float cs = s_clip;
  long lo, hi, a, b;
  chunk_bounds(n, c.world, c.rank, lo, hi);
  cta_slice(lo, hi, a, b);
  bf16* w16 = reinterpret_cast<bf16*>(work16.p[c.rank]);
  for (long i = a + threadIdx.x; i < b; i += blockDim.x) {
    const long k = i - lo;  // index into the shard-local optimizer state
    float mm = m[k], vv = v[k], p = master[i];
    adamw_elem(p, grad[i] * cs, mm, vv, ak);
    m[k] = mm;
    v[k] = vv;
    master[i] = p;
    if (w16) w16[i] = f2bf(p);
  }
  if (!cta_barrier(c, c.epoch + 1)) return;
  for (int kk = 1; kk < c.world; ++kk) {
    const int p = (c.rank + kk) % c.world;
    chunk_bounds(n, c.world, p, lo, hi);
    if (w16 && keep) {
      for (int k = 0; k < nkeep; ++k) {
        const long klo = max(lo, keep[2 * k]), khi = min(hi, keep[2 * k + 1]);
        if (klo >= khi) continue;
        long ka, kb;
        cta_slice(klo, khi, ka, kb);
        copy_range<bf16>(reinterpret_cast<const bf16*>(work16.p[p]), w16, ka, kb);
      }
    }
    cta_slice(lo, hi, a, b);
    if (w16 && !keep) copy_range<bf16>(reinterpret_cast<const bf16*>(work16.p[p]), w16, a, b);
    if (gather_master)
      copy_range<float>(reinterpret_cast<const float*>(master32.p[p]), master, a, b);
  }
  cta_barrier(c, c.epoch + 2);
}
__global__ void __launch_bounds__(kCommThreads)
    zero_adamw_allgather_kernel(CommCtx c, Sigs sq_parts, int nparts, float* master, const float* grad,
                                float* m, float* v, Peers work16, Peers master32, long n, AdamConsts ak,
                                float max_norm, double* sq_out, int gather_master, const long* keep, int nkeep,
                                int* gen_out) {
  DTB_SHARED_COPY(Sigs, s_sq_parts, sq_parts)
  DTB_SHARED_COPY(Peers, s_work16, work16)
  DTB_SHARED_COPY(Peers, s_master32, master32)
  collective_begin(c);
  zero_adamw_allgather_body(c, s_sq_parts, nparts, master, grad, m, v, s_work16, s_master32, n, ak, max_norm, sq_out, gather_master, keep, nkeep, gen_out);
  collective_end(c, 3);
}

// Grid-wide barrier across ranks: returns once every CTA of every rank has arrived
// at `epoch`.  CTA b of rank r publishes slot [b][r] in every rank's signal pad
// (as cta_barrier does) and then polls all gridDim.x * world slots of its own pad.
// Needs every CTA of the grid resident at once (comm grids are at most 128 CTAs of
// 512 threads, four per SM); a CTA that cannot be scheduled makes the others time out.
__device__ bool grid_barrier(const CommCtx& c, uint32_t epoch) {
  __shared__ int failed;
  __syncthreads();
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if (threadIdx.x < c.world) {
    __threadfence_system();
    st_release_sys(c.sp->p[threadIdx.x] + blockIdx.x * kMaxRanks + c.rank, epoch);
  }
  const int slots = (int)gridDim.x * c.world;
  for (int t = threadIdx.x; t < slots; t += blockDim.x) {
    const uint32_t* f = c.sp->p[c.rank] + (t / c.world) * kMaxRanks + (t % c.world);
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
      if ((int)(ld_relaxed_sys(f) - epoch) >= 0) {
        fence_acquire_sys();
        break;
      }
      if (i >= 16u) __nanosleep(128);
      if ((i & 63u) == 0u) {
        if (*reinterpret_cast<volatile int*>(&failed)) break;
        const uint64_t now = globaltimer_ns();
        if (t0 == 0) t0 = now;
        if (group_failed(c) || (t0 != now && now - t0 > c.timeout_ns)) {
          atomicExch(&failed, 1);
          mark_failed(c);
          break;
        }
      }
    }
  }
  __syncthreads();
  return failed == 0;
}

// ZeRO-1 step in ONE kernel: gradient reduce-scatter fused with the global-norm
// clip, the sharded AdamW update and the parameter all-gather (dtrain/zero.py:45-62).
// Phase 1: CTA b sums its slice of this rank's partition over all ranks' fp32
//          gradients in ring order from the owner (bit-equal to dtrain's ring
//          reduce-scatter), scales by 1/W, writes it in place and publishes the
//          slice's fp64 sum of squares in this rank's peer-mapped sq pad.
// Phase 2: grid-wide cross-rank barrier; every CTA then sums all ranks' partials
//          in rank-then-CTA order (the same global norm everywhere) -> clip factor.
// Phase 3: AdamW on the same slice (the CTA reads the gradient it has just
//          written), fp32 master + bf16 working copy.
// Phase 4: per-CTA barrier, then the all-gather of the bf16 working copy (only the
//          `keep` intervals when the forward GEMMs gather the Linear weights) and
//          optionally of the fp32 masters; a last barrier keeps this rank's
//          partition unchanged until every peer has pulled it.
template <int WT>
__device__ __forceinline__ void zero_rs_adamw_body(CommCtx c, const Peers& grads, const Sigs& sq_parts, float* master, float* m, float* v, const Peers& work16,
                         const Peers& master32, long n, AdamConsts ak, float scale, float max_norm, double* sq_out,
                         int gather_master, const long* keep, int nkeep, int* gen_out) {
  __shared__ double red[kCommThreads / 32];
  __shared__ float s_clip;
  if (!cta_enter(c)) return;
  if (gen_out && blockIdx.x == 0 && threadIdx.x == 0) *gen_out = (int)(c.epoch + 1u);
  long lo, hi, a, b;
  chunk_bounds(n, c.world, c.rank, lo, hi);
  cta_slice(lo, hi, a, b);
  float* grad = reinterpret_cast<float*>(grads.p[c.rank]);
  double s = 0.0;
  reduce_range<float, float, WT>(grads, grad, a, b, c.world, c.rank, scale, &s);
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    reinterpret_cast<double*>(sq_parts.p[c.rank])[blockIdx.x] = t;
  }
  if (!grid_barrier(c, c.epoch + 1)) return;
  if (threadIdx.x == 0) {
    double tot = 0.0;
    for (int r = 0; r < c.world; ++r) {
      const double* pp = reinterpret_cast<const double*>(sq_parts.p[r]);
      double rs = 0.0;
      for (int k = 0; k < (int)gridDim.x; ++k) rs += __ldcg(pp + k);
      tot += rs;
    }
    float cs = 1.f;
    const double nrm = sqrt(tot);
    if (max_norm > 0.f && nrm > (double)max_norm && nrm != 0.0) cs = (float)((double)max_norm / (nrm + 1e-6));
    s_clip = cs;
    if (blockIdx.x == 0 && sq_out) sq_out[0] = tot;
  }
  __syncthreads();
  const float cs = s_clip;
  bf16* w16 = reinterpret_cast<bf16*>(work16.p[c.rank]);
  for (long i = a + threadIdx.x; i < b; i += blockDim.x) {
    const long k = i - lo;
    float mm = m[k], vv = v[k], p = master[i];
    adamw_elem(p, grad[i] * cs, mm, vv, ak);
    m[k] = mm;
    v[k] = vv;
    master[i] = p;
    if (w16) w16[i] = f2bf(p);
  }
  if (!cta_barrier(c, c.epoch + 2)) return;
  for (int kk = 1; kk < c.world; ++kk) {
    const int p = (c.rank + kk) % c.world;
    long plo, phi, pa, pb;
    chunk_bounds(n, c.world, p, plo, phi);
    if (w16 && keep) {
      for (int k = 0; k < nkeep; ++k) {
        const long klo = max(plo, keep[2 * k]), khi = min(phi, keep[2 * k + 1]);
        if (klo >= khi) continue;
        long ka, kb;
        cta_slice(klo, khi, ka, kb);
        copy_range<bf16>(reinterpret_cast<const bf16*>(work16.p[p]), w16, ka, kb);
      }
    }
    cta_slice(plo, phi, pa, pb);
    if (w16 && !keep) copy_range<bf16>(reinterpret_cast<const bf16*>(work16.p[p]), w16, pa, pb);
    if (gather_master) copy_range<float>(reinterpret_cast<const float*>(master32.p[p]), master, pa, pb);
  }
  cta_barrier(c, c.epoch + 3);
}
template <int WT>
__global__ void __launch_bounds__(kCommThreads)
    zero_rs_adamw_kernel(CommCtx c, Peers grads, Sigs sq_parts, float* master, float* m, float* v, Peers work16,
                         Peers master32, long n, AdamConsts ak, float scale, float max_norm, double* sq_out,
                         int gather_master, const long* keep, int nkeep, int* gen_out) {
  DTB_SHARED_COPY(Peers, s_grads, grads)
  DTB_SHARED_COPY(Sigs, s_sq_parts, sq_parts)
  DTB_SHARED_COPY(Peers, s_work16, work16)
  DTB_SHARED_COPY(Peers, s_master32, master32)
  collective_begin(c);
  zero_rs_adamw_body<WT>(c, s_grads, s_sq_parts, master, m, v, s_work16, s_master32, n, ak, scale, max_norm, sq_out, gather_master, keep, nkeep, gen_out);
  collective_end(c, 4);
}

// ---------------------------------------------------------------- host side
// Symmetric allocation: cudaMalloc + IPC export.  Returns (ptr, handle bytes).
std::tuple<int64_t, torch::Tensor> symm_alloc(int64_t nbytes) {
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, (size_t)nbytes));
  C10_CUDA_CHECK(cudaMemset(p, 0, (size_t)nbytes));
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  auto t = torch::empty({(int64_t)sizeof(h)}, torch::kUInt8);
  std::memcpy(t.data_ptr(), &h, sizeof(h));
  return {reinterpret_cast<int64_t>(p), t};
}

int64_t symm_open(torch::Tensor handle) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t), "symm_open: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t peer_ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(peer_ptr)); }
void symm_free(int64_t ptr) { cudaFree(reinterpret_cast<void*>(ptr)); }

// A tensor view over raw device memory (no ownership).
torch::Tensor tensor_from_ptr(int64_t ptr, std::vector<int64_t> sizes, c10::ScalarType dtype, int64_t device) {
  auto opts = torch::TensorOptions().dtype(dtype).device(torch::kCUDA, device);
  return torch::from_blob(reinterpret_cast<void*>(ptr), sizes, [](void*) {}, opts);
}

// Host-mapped status word shared by all comm kernels of this process.
static int* g_host_status = nullptr;
static int* g_dev_status = nullptr;
static void ensure_status() {
  if (!g_host_status) {
    C10_CUDA_CHECK(cudaHostAlloc(&g_host_status, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable));
    *g_host_status = 0;
    C10_CUDA_CHECK(cudaHostGetDevicePointer(&g_dev_status, g_host_status, 0));
  }
}
int64_t comm_status() {
  ensure_status();
  return *reinterpret_cast<volatile int*>(g_host_status);
}
void comm_status_clear() {
  ensure_status();
  *reinterpret_cast<volatile int*>(g_host_status) = 0;
}

// Host-side abort of a process group.  comm_abort_prepare() (called when the group is
// made) keeps a pinned word holding 1 and a non-blocking stream; comm_abort() copies
// that word into this rank's "failed" slot (kFailWord of its own signal pad) with the
// copy engine, so collectives that are waiting - including one the calling process is
// blocked on in another thread - see it at their next check and return instead of
// waiting out their timeout.  It also records kStatusAborted for check().
namespace {
std::mutex g_abort_mu;
std::map<int, std::pair<cudaStream_t, uint32_t*>> g_abort;  // device -> (stream, pinned 1)
}  // namespace

void comm_abort_prepare() {
  ensure_status();
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> g(g_abort_mu);
  if (g_abort.count(dev)) return;
  cudaStream_t s;
  C10_CUDA_CHECK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  uint32_t* one = nullptr;
  C10_CUDA_CHECK(cudaHostAlloc(&one, sizeof(uint32_t), cudaHostAllocPortable));
  *one = 1u;
  g_abort[dev] = {s, one};
}

void comm_abort(int64_t own_sig_ptr) {
  TORCH_CHECK(own_sig_ptr != 0, "comm_abort: no signal pad");
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  std::pair<cudaStream_t, uint32_t*> a;
  {
    std::lock_guard<std::mutex> g(g_abort_mu);
    auto it = g_abort.find(dev);
    TORCH_CHECK(it != g_abort.end(), "comm_abort: comm_abort_prepare() was not called on this device");
    a = it->second;
  }
  __atomic_store_n(g_host_status, (int)kStatusAborted, __ATOMIC_SEQ_CST);
  uint32_t* word = reinterpret_cast<uint32_t*>(own_sig_ptr) + kFailWord;
  C10_CUDA_CHECK(cudaMemcpyAsync(word, a.second, sizeof(uint32_t), cudaMemcpyHostToDevice, a.first));
  C10_CUDA_CHECK(cudaStreamSynchronize(a.first));
}

// Descriptor of a collective: its kind, element count and dtype, mixed into 32 bits.
static uint32_t op_tag(uint32_t kind, int64_t n, int64_t dtype) {
  uint64_t h = (uint64_t)n * 0x9E3779B97F4A7C15ull;
  h ^= (uint64_t)kind << 56 ^ (uint64_t)dtype << 48;
  h ^= h >> 29;
  return (uint32_t)(h ^ (h >> 32));
}

static CommCtx make_ctx(const std::vector<int64_t>& sigs, int64_t rank, double timeout_s, uint32_t tag) {
  ensure_status();
  CommCtx c{};
  const int W = (int)sigs.size();
  TORCH_CHECK(W >= 1 && W <= kMaxRanks, "comm: world size must be 1..8");
  TORCH_CHECK(rank >= 0 && rank < W, "comm: bad rank");
  for (int i = 0; i < W; ++i) c.sig.p[i] = reinterpret_cast<uint32_t*>(sigs[i]);
  c.rank = (int)rank;
  c.world = W;
  c.epoch = 0;  // read from the rank's epoch counter by collective_begin()
  c.tag = tag;
  c.timeout_ns = (uint64_t)(timeout_s * 1e9);
  c.host_status = g_dev_status;
  return c;
}

static Peers make_peers(const std::vector<int64_t>& ptrs, int64_t byte_offset) {
  Peers p{};
  for (size_t i = 0; i < ptrs.size(); ++i) p.p[i] = reinterpret_cast<char*>(ptrs[i]) + byte_offset;
  return p;
}

// A lean kernel's CTAs must be able to share an SM with a GEMM CTA that uses
// ~226 KB of shared memory.  An SM's L1/shared split is set for the CTAs it runs,
// and a kernel with almost no shared memory would by default get a small shared
// carve-out - a GEMM CTA then cannot join that SM until the comm CTA leaves.  So
// lean kernels ask for the maximum shared carve-out (once per kernel).
template <typename K>
static void prefer_max_shared(K* kern) {
  static bool done = false;
  if (!done) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                        (int)cudaSharedmemCarveoutMaxShared));
    done = true;
  }
}

// Device-side timestamps for tracing a step: one thread writes %globaltimer (ns,
// the same clock on every SM) into buf[slot] when the stream reaches it.
__global__ void stamp_kernel(int64_t* slot) { *slot = (int64_t)globaltimer_ns(); }

void stamp(torch::Tensor buf, int64_t slot) {
  TORCH_CHECK(buf.is_cuda() && buf.scalar_type() == at::kLong && slot >= 0 && slot < buf.numel(),
              "stamp: int64 CUDA buffer and a slot inside it");
  stamp_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream()>>>(buf.data_ptr<int64_t>() + slot);
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// CTAs of a full-width collective: ~64 KB per CTA, at most 64 CTAs, unless the
// caller asks for a count.
static int comm_blocks(long bytes, int64_t want) {
  if (want > 0) return (int)std::min<int64_t>(want, kMaxCommBlocks);
  const long per = 64 * 1024;
  return (int)std::max<long>(1, std::min<long>(64, (bytes + per - 1) / per));
}

// CTAs of a lean collective (one 128-thread CTA beside each SM's resident
// kernel): ~16 KB per CTA, at most one per SM.
static int lean_blocks(long bytes, int64_t want) {
  if (want > 0) return (int)std::min<int64_t>(want, kMaxCommBlocks);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long per = 16 * 1024;
  return (int)std::max<long>(1, std::min<long>(std::min(sms, kMaxCommBlocks), (bytes + per - 1) / per));
}

int64_t collective_blocks(int64_t nbytes, int64_t want, bool lean) {
  return lean ? lean_blocks(nbytes, want) : comm_blocks(nbytes, want);
}

static SqOut make_sq(const std::vector<int64_t>& pads, int64_t base, int64_t stride, int W, int nb) {
  SqOut s{};
  if (pads.empty()) return s;
  TORCH_CHECK((int)pads.size() == W, "allreduce: one sum-of-squares pad per rank expected");
  TORCH_CHECK(base >= 0 && stride > 0 && base + nb <= stride, "allreduce: sum-of-squares slots [", base, ", ",
              base + nb, ") exceed the per-rank stride ", stride);
  for (int i = 0; i < W; ++i) s.p[i] = reinterpret_cast<double*>(pads[i]);
  s.base = (int)base;
  s.stride = (int)stride;
  return s;
}

// Every collective launches one kernel on the current stream and returns its CTA
// count.  Flag epochs come from the device counter (see collective_begin).
int64_t allreduce(std::vector<int64_t> sigs, int64_t rank, std::vector<int64_t> bufs, int64_t byte_offset, int64_t n,
                  int64_t in_dtype, int64_t out_ptr, int64_t out_dtype, int64_t algo, int64_t order, double scale,
                  double timeout_s, int64_t blocks, bool lean, std::vector<int64_t> sq_pads, int64_t sq_base,
                  int64_t sq_stride) {
  CommCtx c = make_ctx(sigs, rank, timeout_s, op_tag(1 + (uint32_t)algo, n, in_dtype * 8 + out_dtype));
  Peers in = make_peers(bufs, byte_offset);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const long esz = in_dtype == DT_F32 ? 4 : 2;
  const int nb = lean ? lean_blocks(n * esz, blocks) : comm_blocks(n * esz, blocks);
  if (algo == 0) {  // one-shot, out-of-place
    TORCH_CHECK(out_ptr != 0, "allreduce one-shot needs an output buffer");
    TORCH_CHECK(!lean && sq_pads.empty(), "allreduce one-shot: no lean variant and no sum of squares");
    const int od = (int)order;
    const float sc = (float)scale;
    if (in_dtype == DT_F32 && out_dtype == DT_F32) {
      auto* o = reinterpret_cast<float*>(out_ptr);
      switch (c.world) {
        case 2: allreduce_oneshot_kernel<float, float, 2><<<nb, kCommThreads, 0, st>>>(c, in, o, n, od, sc); break;
        case 4: allreduce_oneshot_kernel<float, float, 4><<<nb, kCommThreads, 0, st>>>(c, in, o, n, od, sc); break;
        case 8: allreduce_oneshot_kernel<float, float, 8><<<nb, kCommThreads, 0, st>>>(c, in, o, n, od, sc); break;
        default: allreduce_oneshot_kernel<float, float, 0><<<nb, kCommThreads, 0, st>>>(c, in, o, n, od, sc);
      }
    } else if (in_dtype == DT_BF16 && out_dtype == DT_F32)
      allreduce_oneshot_kernel<bf16, float, 0><<<nb, kCommThreads, 0, st>>>(c, in, reinterpret_cast<float*>(out_ptr), n, od, sc);
    else if (in_dtype == DT_BF16 && out_dtype == DT_BF16)
      allreduce_oneshot_kernel<bf16, bf16, 0><<<nb, kCommThreads, 0, st>>>(c, in, reinterpret_cast<bf16*>(out_ptr), n, od, sc);
    else
      TORCH_CHECK(false, "allreduce: unsupported dtype pair");
    count_launch();
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return nb;
  }
  TORCH_CHECK(in_dtype == out_dtype, "allreduce two-shot: in/out dtypes must match");
  void* out = out_ptr ? reinterpret_cast<void*>(out_ptr) : in.p[rank];
  const SqOut sq = make_sq(sq_pads, sq_base, sq_stride, c.world, nb);
  const int od = (int)order;
  const float sc = (float)scale;
  const int nt = lean ? kLeanThreads : kCommThreads;
#define DTB_TWOSHOT(T, WTV, LN)                                                           \
  do {                                                                                    \
    if (LN) prefer_max_shared(allreduce_twoshot_kernel<T, WTV, LN>);                      \
    allreduce_twoshot_kernel<T, WTV, LN><<<nb, nt, 0, st>>>(c, in, reinterpret_cast<T*>(out), n, od, sc, sq); \
  } while (0)
  if (in_dtype == DT_F32) {
    if (lean) {
      switch (c.world) {
        case 2: DTB_TWOSHOT(float, 2, true); break;
        case 4: DTB_TWOSHOT(float, 4, true); break;
        case 8: DTB_TWOSHOT(float, 8, true); break;
        default: DTB_TWOSHOT(float, 0, true);
      }
    } else {
      switch (c.world) {
        case 2: DTB_TWOSHOT(float, 2, false); break;
        case 4: DTB_TWOSHOT(float, 4, false); break;
        case 8: DTB_TWOSHOT(float, 8, false); break;
        default: DTB_TWOSHOT(float, 0, false);
      }
    }
  } else if (lean) {
    switch (c.world) {
      case 2: DTB_TWOSHOT(bf16, 2, true); break;
      case 4: DTB_TWOSHOT(bf16, 4, true); break;
      case 8: DTB_TWOSHOT(bf16, 8, true); break;
      default: DTB_TWOSHOT(bf16, 0, true);
    }
  } else {
    switch (c.world) {
      case 2: DTB_TWOSHOT(bf16, 2, false); break;
      case 4: DTB_TWOSHOT(bf16, 4, false); break;
      case 8: DTB_TWOSHOT(bf16, 8, false); break;
      default: DTB_TWOSHOT(bf16, 0, false);
    }
  }
#undef DTB_TWOSHOT
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return nb;
}

// All-reduce through the switch (see allreduce_nvls_kernel): `mc_ptr` is the
// multicast address of the buffer that holds the data at `byte_offset`.
int64_t allreduce_nvls(std::vector<int64_t> sigs, int64_t rank, int64_t mc_ptr, int64_t byte_offset, int64_t n,
                       int64_t dtype, double scale, double timeout_s, int64_t blocks, bool lean,
                       std::vector<int64_t> sq_pads, int64_t sq_base, int64_t sq_stride) {
  TORCH_CHECK(mc_ptr != 0, "allreduce_nvls: the buffer has no multicast mapping");
  TORCH_CHECK(dtype == DT_F32 ? (mc_ptr + byte_offset) % 4 == 0 : ((mc_ptr + byte_offset) % 16 == 0 && n % 8 == 0),
              "allreduce_nvls: fp32 data must be 4-byte aligned; bf16 data must start on a 16-byte boundary and "
              "hold a multiple of 8 elements");
  CommCtx c = make_ctx(sigs, rank, timeout_s, op_tag(8, n, dtype));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const long nbytes = n * (dtype == DT_F32 ? 4 : 2);
  const int nb = lean ? lean_blocks(nbytes, blocks) : comm_blocks(nbytes, blocks);
  const SqOut sq = make_sq(sq_pads, sq_base, sq_stride, c.world, nb);
  char* mc = reinterpret_cast<char*>(mc_ptr) + byte_offset;
  const float sc = (float)scale;
  if (lean) {
    if (dtype == DT_F32) {
      prefer_max_shared(allreduce_nvls_kernel<float, true>);
      allreduce_nvls_kernel<float, true><<<nb, kLeanThreads, 0, st>>>(c, mc, n, sc, sq);
    } else {
      prefer_max_shared(allreduce_nvls_kernel<bf16, true>);
      allreduce_nvls_kernel<bf16, true><<<nb, kLeanThreads, 0, st>>>(c, mc, n, sc, sq);
    }
  } else if (dtype == DT_F32) {
    allreduce_nvls_kernel<float, false><<<nb, kCommThreads, 0, st>>>(c, mc, n, sc, sq);
  } else {
    allreduce_nvls_kernel<bf16, false><<<nb, kCommThreads, 0, st>>>(c, mc, n, sc, sq);
  }
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return nb;
}

// Reduce-scatter (fp32) through the switch into this rank's partition of `out_ptr`.
int64_t reduce_scatter_nvls(std::vector<int64_t> sigs, int64_t rank, int64_t mc_ptr, int64_t byte_offset, int64_t n,
                            int64_t out_ptr, double scale, int64_t sq_part_ptr, double timeout_s, int64_t blocks) {
  TORCH_CHECK(mc_ptr != 0 && out_ptr != 0 && (mc_ptr + byte_offset) % 16 == 0 && out_ptr % 16 == 0,
              "reduce_scatter_nvls: 16-byte aligned multicast data and output expected");
  CommCtx c = make_ctx(sigs, rank, timeout_s, op_tag(9, n, DT_F32));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int nb = comm_blocks(n * 4, blocks);
  reduce_scatter_nvls_kernel<<<nb, kCommThreads, 0, st>>>(c, reinterpret_cast<const char*>(mc_ptr) + byte_offset,
                                                          reinterpret_cast<float*>(out_ptr), n, (float)scale,
                                                          reinterpret_cast<double*>(sq_part_ptr));
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return nb;
}

void sq_total(torch::Tensor pad, torch::Tensor out, int64_t world, int64_t stride, int64_t lo, int64_t hi) {
  TORCH_CHECK(pad.is_cuda() && pad.scalar_type() == at::kDouble && pad.is_contiguous(), "sq_total: fp64 CUDA pad");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kDouble && out.numel() >= 1, "sq_total: fp64 CUDA out");
  TORCH_CHECK(world >= 1 && 0 <= lo && lo < hi && hi <= stride && world * stride <= pad.numel(),
              "sq_total: slots [", lo, ", ", hi, ") x ", world, " ranks do not fit a pad of ", pad.numel());
  sq_total_kernel<<<1, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(pad.data_ptr<double>(), (int)world, stride, lo,
                                                                     hi, out.data_ptr<double>());
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t reduce_scatter(std::vector<int64_t> sigs, int64_t rank, std::vector<int64_t> bufs,
                       int64_t byte_offset, int64_t n, int64_t dtype, int64_t out_ptr, int64_t order, double scale,
                       int64_t sq_part_ptr, double timeout_s, int64_t blocks) {
  CommCtx c = make_ctx(sigs, rank, timeout_s, op_tag(4, n, dtype));
  Peers in = make_peers(bufs, byte_offset);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int nb = comm_blocks(n * (dtype == DT_F32 ? 4 : 2), blocks);
  void* out = out_ptr ? reinterpret_cast<void*>(out_ptr) : in.p[rank];
  double* sq = reinterpret_cast<double*>(sq_part_ptr);
  if (dtype == DT_F32) {
    auto* o = reinterpret_cast<float*>(out);
    const int od = (int)order;
    const float sc = (float)scale;
    switch (c.world) {
      case 2: reduce_scatter_kernel<float, float, 2><<<nb, kCommThreads, 0, st>>>(c, in, o, n, od, sc, sq); break;
      case 4: reduce_scatter_kernel<float, float, 4><<<nb, kCommThreads, 0, st>>>(c, in, o, n, od, sc, sq); break;
      case 8: reduce_scatter_kernel<float, float, 8><<<nb, kCommThreads, 0, st>>>(c, in, o, n, od, sc, sq); break;
      default: reduce_scatter_kernel<float, float, 0><<<nb, kCommThreads, 0, st>>>(c, in, o, n, od, sc, sq);
    }
  } else {
    auto* o = reinterpret_cast<bf16*>(out);
    const int od = (int)order;
    const float sc = (float)scale;
    switch (c.world) {
      case 2: reduce_scatter_kernel<bf16, bf16, 2><<<nb, kCommThreads, 0, st>>>(c, in, o, n, od, sc, sq); break;
      case 4: reduce_scatter_kernel<bf16, bf16, 4><<<nb, kCommThreads, 0, st>>>(c, in, o, n, od, sc, sq); break;
      case 8: reduce_scatter_kernel<bf16, bf16, 8><<<nb, kCommThreads, 0, st>>>(c, in, o, n, od, sc, sq); break;
      default: reduce_scatter_kernel<bf16, bf16, 0><<<nb, kCommThreads, 0, st>>>(c, in, o, n, od, sc, sq);
    }
  }
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return nb;
}

int64_t all_gather(std::vector<int64_t> sigs, int64_t rank, std::vector<int64_t> bufs,
                   int64_t byte_offset, int64_t n, int64_t dtype, double timeout_s, int64_t blocks) {
  CommCtx c = make_ctx(sigs, rank, timeout_s, op_tag(5, n, dtype));
  Peers in = make_peers(bufs, byte_offset);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int nb = comm_blocks(n * (dtype == DT_F32 ? 4 : 2), blocks);
  if (dtype == DT_F32)
    all_gather_kernel<float><<<nb, kCommThreads, 0, st>>>(c, in, reinterpret_cast<float*>(in.p[rank]), n);
  else
    all_gather_kernel<bf16><<<nb, kCommThreads, 0, st>>>(c, in, reinterpret_cast<bf16*>(in.p[rank]), n);
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return nb;
}

int64_t broadcast(std::vector<int64_t> sigs, int64_t rank, std::vector<int64_t> bufs,
                  int64_t byte_offset, int64_t nbytes, int64_t root, int64_t cast_src, int64_t out16, int64_t n16,
                  double timeout_s, int64_t blocks) {
  CommCtx c = make_ctx(sigs, rank, timeout_s, op_tag(6, nbytes, root));
  Peers in = make_peers(bufs, byte_offset);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int nb = comm_blocks(nbytes, blocks);
  broadcast_kernel<<<nb, kCommThreads, 0, st>>>(c, in, in.p[rank], nbytes, (int)root,
                                                reinterpret_cast<const float*>(cast_src),
                                                reinterpret_cast<bf16*>(out16), n16);
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return nb;
}

int64_t device_barrier(std::vector<int64_t> sigs, int64_t rank, double timeout_s) {
  CommCtx c = make_ctx(sigs, rank, timeout_s, op_tag(7, 0, 0));
  const int nb = 1;
  barrier_kernel<<<nb, 32, 0, at::cuda::getCurrentCUDAStream()>>>(c);
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return nb;
}

int64_t zero_adamw_allgather(std::vector<int64_t> sigs, int64_t rank, std::vector<int64_t> sq_parts,
                             int64_t nparts, torch::Tensor master, torch::Tensor grad, torch::Tensor m,
                             torch::Tensor v, std::vector<int64_t> work16, std::vector<int64_t> master32, int64_t n,
                             double lr, double b1, double b2, double eps, double wd, int64_t t, double max_norm,
                             c10::optional<torch::Tensor> sq_out, bool gather_master, double timeout_s,
                             int64_t blocks, c10::optional<torch::Tensor> keep, c10::optional<torch::Tensor> gen_word) {
  const int64_t nkeep_tag = (keep && keep->defined()) ? keep->size(0) + 1 : 0;
  CommCtx c = make_ctx(sigs, rank, timeout_s, op_tag(8, n, (gather_master ? 1 : 0) + 2 * nkeep_tag));
  Sigs sp{};
  for (size_t i = 0; i < sq_parts.size(); ++i) sp.p[i] = reinterpret_cast<uint32_t*>(sq_parts[i]);
  Peers w16 = make_peers(work16, 0), m32 = make_peers(master32, 0);
  const AdamConsts ak = adam_consts(lr, b1, b2, eps, wd, t);
  double* sqo = (sq_out && sq_out->defined()) ? sq_out->data_ptr<double>() : nullptr;
  const long* kp = nullptr;
  int nkeep = 0;
  if (keep && keep->defined()) {
    TORCH_CHECK(keep->is_cuda() && keep->scalar_type() == at::kLong && keep->is_contiguous() && keep->dim() == 2 &&
                    keep->size(1) == 2,
                "zero_adamw_allgather: keep must be a [k, 2] int64 CUDA tensor");
    kp = keep->data_ptr<int64_t>();
    nkeep = (int)keep->size(0);
  }
  int* gw = nullptr;
  if (gen_word && gen_word->defined()) {
    TORCH_CHECK(gen_word->is_cuda() && gen_word->scalar_type() == at::kInt, "zero_adamw_allgather: gen_word int32");
    gw = gen_word->data_ptr<int>();
  }
  const int nb = comm_blocks(n * 2, blocks);
  zero_adamw_allgather_kernel<<<nb, kCommThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      c, sp, (int)nparts, master.data_ptr<float>(), grad.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
      w16, m32, n, ak, (float)max_norm, sqo, gather_master ? 1 : 0, kp, nkeep, gw);
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return nb;
}

// One-kernel ZeRO-1 step (zero_rs_adamw_kernel).  `grads` are every rank's
// addresses of the flat fp32 gradient, `sq_parts` every rank's fp64 pad of at least
// `blocks` (or 64) slots.  Returns the CTA count.
int64_t zero_rs_adamw(std::vector<int64_t> sigs, int64_t rank, std::vector<int64_t> grads,
                      std::vector<int64_t> sq_parts, torch::Tensor master, torch::Tensor m, torch::Tensor v,
                      std::vector<int64_t> work16, std::vector<int64_t> master32, int64_t n, double lr, double b1,
                      double b2, double eps, double wd, int64_t t, double scale, double max_norm,
                      c10::optional<torch::Tensor> sq_out, bool gather_master, double timeout_s, int64_t blocks,
                      c10::optional<torch::Tensor> keep, c10::optional<torch::Tensor> gen_word) {
  const int64_t nkeep_tag = (keep && keep->defined()) ? keep->size(0) + 1 : 0;
  CommCtx c = make_ctx(sigs, rank, timeout_s, op_tag(9, n, (gather_master ? 1 : 0) + 2 * nkeep_tag));
  TORCH_CHECK(grads.size() == sigs.size() && sq_parts.size() == sigs.size(), "zero_rs_adamw: one pointer per rank");
  Sigs sp{};
  for (size_t i = 0; i < sq_parts.size(); ++i) sp.p[i] = reinterpret_cast<uint32_t*>(sq_parts[i]);
  Peers g = make_peers(grads, 0), w16 = make_peers(work16, 0), m32 = make_peers(master32, 0);
  const AdamConsts ak = adam_consts(lr, b1, b2, eps, wd, t);
  double* sqo = (sq_out && sq_out->defined()) ? sq_out->data_ptr<double>() : nullptr;
  const long* kp = nullptr;
  int nkeep = 0;
  if (keep && keep->defined()) {
    TORCH_CHECK(keep->is_cuda() && keep->scalar_type() == at::kLong && keep->is_contiguous() && keep->dim() == 2 &&
                    keep->size(1) == 2,
                "zero_rs_adamw: keep must be a [k, 2] int64 CUDA tensor");
    kp = keep->data_ptr<int64_t>();
    nkeep = (int)keep->size(0);
  }
  int* gw = nullptr;
  if (gen_word && gen_word->defined()) {
    TORCH_CHECK(gen_word->is_cuda() && gen_word->scalar_type() == at::kInt, "zero_rs_adamw: gen_word int32");
    gw = gen_word->data_ptr<int>();
  }
  const int nb = comm_blocks(n * 4, blocks);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  float* mp = master.data_ptr<float>();
  float* mm = m.data_ptr<float>();
  float* vp = v.data_ptr<float>();
  const float sc = (float)scale, mn = (float)max_norm;
  const int gm = gather_master ? 1 : 0;
#define DTB_ZRA(WTV)                                                                                             \
  zero_rs_adamw_kernel<WTV><<<nb, kCommThreads, 0, st>>>(c, g, sp, mp, mm, vp, w16, m32, n, ak, sc, mn, sqo, gm, kp, \
                                                         nkeep, gw)
  switch (c.world) {
    case 2: DTB_ZRA(2); break;
    case 4: DTB_ZRA(4); break;
    case 8: DTB_ZRA(8); break;
    default: DTB_ZRA(0);
  }
#undef DTB_ZRA
  count_launch();
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return nb;
}

// Native per-group state so a collective on a peer-mapped tensor costs one call
// from Python: the registered buffers (every rank's base pointer), the signal
// pads and the timeout live here (the flag epoch counter lives on the device).
CommEngine::CommEngine(int64_t rank, int64_t world, std::vector<int64_t> sigs, double timeout_s, int64_t blocks)
    : rank_(rank), world_(world), sigs_(std::move(sigs)), timeout_(timeout_s), blocks_(blocks) {}

static int64_t dt_code(const torch::Tensor& t) {
  if (t.scalar_type() == at::kFloat) return DT_F32;
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, "NVLink collectives support float32 and bfloat16");
  return DT_BF16;
}

int64_t CommEngine::register_buffer(std::vector<int64_t> ptrs, int64_t nbytes, int64_t mc_ptr) {
  TORCH_CHECK((int64_t)ptrs.size() == world_, "register_buffer: one pointer per rank expected");
  bufs_.push_back(std::move(ptrs));
  sizes_.push_back(nbytes);
  mcs_.push_back(mc_ptr);
  return (int64_t)bufs_.size() - 1;
}

void CommEngine::forget_buffers() {
  bufs_.clear();
  sizes_.clear();
  mcs_.clear();
}

bool CommEngine::has_multicast(torch::Tensor t) const {
  int64_t id, off;
  return locate(t, id, off) && mcs_[id] != 0;
}

int64_t CommEngine::allreduce_nvls(torch::Tensor t, double scale, int64_t blocks, bool lean,
                                   c10::optional<torch::Tensor> sq_pad, int64_t sq_base, int64_t sq_stride) {
  int64_t id, off;
  TORCH_CHECK(t.is_contiguous() && locate(t, id, off) && mcs_[id] != 0,
              "allreduce_nvls: tensor is not in a multicast-mapped buffer");
  std::vector<int64_t> pads;
  if (sq_pad && sq_pad->defined()) {
    TORCH_CHECK(sq_pad->scalar_type() == at::kDouble, "allreduce_nvls: the sum-of-squares pad must be fp64");
    pads = peer_ptrs(*sq_pad);
    TORCH_CHECK(sq_pad->numel() >= world_ * sq_stride, "allreduce_nvls: sum-of-squares pad too small");
  }
  ++issued_;
  return dtb::allreduce_nvls(sigs_, rank_, mcs_[id], off, t.numel(), dt_code(t), scale, timeout_,
                             blocks > 0 ? blocks : blocks_, lean, pads, sq_base, sq_stride);
}

torch::Tensor CommEngine::reduce_scatter_nvls(torch::Tensor flat, double scale, int64_t sq_part_ptr, int64_t blocks) {
  int64_t id, off;
  TORCH_CHECK(flat.is_contiguous() && flat.scalar_type() == at::kFloat && locate(flat, id, off) && mcs_[id] != 0,
              "reduce_scatter_nvls: fp32 tensor in a multicast-mapped buffer expected");
  ++issued_;
  dtb::reduce_scatter_nvls(sigs_, rank_, mcs_[id], off, flat.numel(), reinterpret_cast<int64_t>(flat.data_ptr()),
                           scale, sq_part_ptr, timeout_, blocks > 0 ? blocks : blocks_);
  const int64_t n = flat.numel(), base = n / world_, extra = n % world_;
  const int64_t lo = rank_ * base + std::min(rank_, extra);
  return flat.narrow(0, lo, base + (rank_ < extra ? 1 : 0));
}

bool CommEngine::locate(const torch::Tensor& t, int64_t& id, int64_t& off) const {
  const int64_t p = reinterpret_cast<int64_t>(t.data_ptr());
  const int64_t nb = t.numel() * (int64_t)t.element_size();
  for (size_t i = 0; i < bufs_.size(); ++i) {
    const int64_t base = bufs_[i][rank_];
    if (p >= base && p + nb <= base + sizes_[i]) {
      id = (int64_t)i;
      off = p - base;
      return true;
    }
  }
  return false;
}

bool CommEngine::contains(torch::Tensor t) const {
  int64_t id, off;
  return locate(t, id, off);
}

int64_t CommEngine::allreduce_inplace(torch::Tensor t, int64_t order, double scale, int64_t blocks, bool lean,
                                      c10::optional<torch::Tensor> sq_pad, int64_t sq_base, int64_t sq_stride) {
  int64_t id, off;
  TORCH_CHECK(t.is_contiguous() && locate(t, id, off), "allreduce_inplace: tensor is not in a registered buffer");
  std::vector<int64_t> pads;
  if (sq_pad && sq_pad->defined()) {
    TORCH_CHECK(sq_pad->scalar_type() == at::kDouble, "allreduce_inplace: the sum-of-squares pad must be fp64");
    pads = peer_ptrs(*sq_pad);
    TORCH_CHECK(sq_pad->numel() >= world_ * sq_stride, "allreduce_inplace: sum-of-squares pad too small");
  }
  ++issued_;
  return dtb::allreduce(sigs_, rank_, bufs_[id], off, t.numel(), dt_code(t), 0, dt_code(t), 1, order, scale, timeout_,
                        blocks > 0 ? blocks : blocks_, lean, pads, sq_base, sq_stride);
}

int64_t CommEngine::device_epoch() const {
  uint32_t v = 0;
  C10_CUDA_CHECK(cudaMemcpy(&v, reinterpret_cast<const uint32_t*>(sigs_[rank_]) + kCtrWord, sizeof(v),
                            cudaMemcpyDeviceToHost));
  return (int64_t)v;
}

torch::Tensor CommEngine::reduce_scatter(torch::Tensor flat, int64_t order, double scale, int64_t sq_part_ptr,
                                         int64_t blocks) {
  int64_t id, off;
  TORCH_CHECK(flat.is_contiguous() && locate(flat, id, off), "reduce_scatter: tensor is not in a registered buffer");
  ++issued_;
  dtb::reduce_scatter(sigs_, rank_, bufs_[id], off, flat.numel(), dt_code(flat), 0, order, scale, sq_part_ptr, timeout_,
                      blocks > 0 ? blocks : blocks_);
  const int64_t n = flat.numel(), base = n / world_, extra = n % world_;
  const int64_t lo = rank_ * base + std::min(rank_, extra);
  return flat.narrow(0, lo, base + (rank_ < extra ? 1 : 0));
}

void CommEngine::all_gather(torch::Tensor flat) {
  int64_t id, off;
  TORCH_CHECK(flat.is_contiguous() && locate(flat, id, off), "all_gather: tensor is not in a registered buffer");
  ++issued_;
  dtb::all_gather(sigs_, rank_, bufs_[id], off, flat.numel(), dt_code(flat), timeout_, blocks_);
}

void CommEngine::barrier() {
  ++issued_;
  dtb::device_barrier(sigs_, rank_, timeout_);
}

std::vector<int64_t> CommEngine::peer_ptrs(torch::Tensor t) const {
  int64_t id, off;
  TORCH_CHECK(locate(t, id, off), "peer_ptrs: tensor is not in a registered buffer");
  std::vector<int64_t> out(bufs_[id]);
  for (auto& p : out) p += off;
  return out;
}

int64_t comm_max_blocks() { return kMaxCommBlocks; }
int64_t comm_max_ranks() { return kMaxRanks; }

DTB_DEFINE_STATUS_READER(status_comm)

}  // namespace dtb
