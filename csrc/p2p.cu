// Peer-to-peer collectives over NVLink / NVSwitch for the sharded (zero) data-parallel mode: buffers allocated with
// cudaMalloc and shared between the ranks of one node by CUDA IPC, and kernels that move data with plain stores into
// peer memory and synchronise with epoch flags (bounded waits; no NCCL on these paths).
//
// Reduce-scatter of one gradient bucket (the bucket is [W owner segments of `seg` fp32]):
//   push kernel    rank r writes its segment for owner o into o's receive buffer slot r (for every o != r), after o
//                  has acknowledged the previous epoch's data in that slot; the last CTA then raises flag[r][b] = epoch
//                  in every owner's flag array (release, system scope).
//   reduce kernel  the owner waits for flag[r][b] >= epoch from every r, sums its own segment and the W - 1 received
//                  segments in rank order (deterministic), writes the sum in place and a per-CTA sum of squares (the
//                  global-norm clip), and the last CTA acknowledges the epoch to every sender.
// The push kernel never waits for anything the same step produces, so the reduce kernel's waits always resolve,
// whatever the number of resident CTAs. Weight broadcast: every owner writes its bf16 segment of a bucket into every
// peer's compute-weight buffer and raises a flag; the consumer waits for all flags before the next forward.
// Reference: the NCCL reduce-scatter / all-gather of the reference's FSDP2 path (baselines/PixelGen/src/utils/
// fsdp_setup.py:116-148); this is the same data movement as plain NVLink stores.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "status.h"

namespace ng {

#ifndef NG_PEER_WAIT_NS
#define NG_PEER_WAIT_NS 60000000000ull  // a peer may legitimately be far behind (first steps, stragglers): 60 s
#endif

struct PeerTable {
  int64_t p[8];  // device addresses of the same buffer on ranks 0..W-1 (this rank's own address at [rank])
};

__device__ __forceinline__ long long ld_acquire_sys(const long long* p) {
  long long v;
  asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(long long* p, long long v) {
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// waits (bounded by budget_ns) until *flag >= epoch; returns false and raises an error on timeout
__device__ bool wait_flag(const long long* flag, long long epoch, int* err,
                          unsigned long long budget_ns = NG_PEER_WAIT_NS) {
  if (ld_acquire_sys(flag) >= epoch) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t n = 0;
  while (ld_acquire_sys(flag) < epoch) {
    if ((++n & 1023u) == 0 && globaltimer_ns() - t0 > budget_ns) {
      raise_error(err, kErrPeerFlag);
      return false;
    }
  }
  return true;
}

// Completion of a grid: every CTA adds 1 to the counter, plus kFailBit when its waits gave up (or the status word
// already held an error). The CTA whose add completes the grid resets the counter and learns whether any CTA failed;
// only then may it publish a flag or an acknowledgement. A rank whose wait timed out therefore never tells its peers
// that data is there when it is not: they time out in turn and report on their own status words, instead of reading
// slots that were never written.
constexpr unsigned int kFailBit = 1u << 20;  // grids here have at most 2 x 148 CTAs, far below 2^20

// returns true in the one thread (threadIdx.x == 0 of the last CTA) that must publish, false everywhere else
__device__ __forceinline__ bool grid_done_ok(unsigned int* counter, bool cta_ok) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x != 0) return false;
  const unsigned int prev = atomicAdd(counter, 1u + (cta_ok ? 0u : kFailBit));
  if ((prev & (kFailBit - 1)) != gridDim.x - 1) return false;
  *counter = 0;
  __threadfence_system();
  return cta_ok && (prev >> 20) == 0;
}

__device__ __forceinline__ bool status_clean(const int* err) {
  return *reinterpret_cast<const volatile int*>(err) == 0;
}

// flags / acks arrays are [W][nb] int64 on every rank: entry [r][b] on rank o = the last epoch of bucket b that rank
// r pushed to o (flags) / that owner r consumed from o (acks).
__global__ void __launch_bounds__(256) p2p_push_kernel(const float* __restrict__ grad, PeerTable recv, PeerTable flags,
                                                       long long* __restrict__ acks, unsigned int* counter, int W,
                                                       int rank, int nb, int b, int64_t start, int64_t seg,
                                                       long long epoch, int* err) {
  // 1) every owner consumed the previous epoch of this bucket (its slot for us may be overwritten)
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    for (int o = 0; o < W; ++o)
      if (o != rank && !wait_flag(acks + (int64_t)o * nb + b, epoch - 1, err)) ok = 0;
  }
  __syncthreads();
  if (ok) {
    // 2) our segment for owner o -> o's receive slot `rank`, as float4 stores into peer memory. Work unit = one
    //    warp's 512 contiguous bytes for one owner; consecutive units rotate over the owners, starting after this
    //    rank, so every receiver takes data from all senders at once instead of all senders targeting one owner.
    const int64_t n4 = seg / 4;
    const int64_t nchunk = (n4 + 31) / 32;
    const int64_t units = (int64_t)(W - 1) * nchunk;
    const int lane = threadIdx.x & 31;
    const int64_t wpb = blockDim.x >> 5;
    for (int64_t u = blockIdx.x * wpb + (threadIdx.x >> 5); u < units; u += gridDim.x * wpb) {
      const int o = (rank + 1 + (int)(u % (W - 1))) % W;
      const int64_t j = (u / (W - 1)) * 32 + lane;
      if (j < n4) {
        const float4* src = reinterpret_cast<const float4*>(grad + start + (int64_t)o * seg) + j;
        float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(recv.p[o]) + start + (int64_t)rank * seg) + j;
        *dst = *src;
      }
    }
  }
  // 3) the last CTA raises our flag for this bucket at every owner (after everyone's stores are visible), unless some
  //    CTA gave up its wait and moved no data
  if (grid_done_ok(counter, ok != 0))
    for (int o = 0; o < W; ++o)
      if (o != rank) st_release_sys(reinterpret_cast<long long*>(flags.p[o]) + (int64_t)rank * nb + b, epoch);
}

__global__ void __launch_bounds__(256) p2p_reduce_kernel(float* __restrict__ grad, const float* __restrict__ recv,
                                                         const long long* __restrict__ flags, PeerTable acks,
                                                         unsigned int* counter, float* __restrict__ sumsq, int W,
                                                         int rank, int nb, int b, int64_t start, int64_t seg,
                                                         long long epoch, int* err) {
  __shared__ int ok;
  __shared__ float red[8];
  if (threadIdx.x == 0) {
    ok = 1;
    for (int r = 0; r < W; ++r)
      if (r != rank && !wait_flag(flags + (int64_t)r * nb + b, epoch, err)) ok = 0;
  }
  __syncthreads();
  float sq = 0.f;
  if (ok) {
    const int64_t n4 = seg / 4;
    float4* mine = reinterpret_cast<float4*>(grad + start + (int64_t)rank * seg);
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n4; j += (int64_t)gridDim.x * blockDim.x) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < W; ++r) {  // rank order: the same sum on every run
        const float4 v = r == rank ? mine[j] : reinterpret_cast<const float4*>(recv + start + (int64_t)r * seg)[j];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      mine[j] = acc;
      sq += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
    }
  }
  // per-CTA partial of the sum of squares (summed in CTA order by the host side: deterministic)
  sq = warp_sum(sq);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    sumsq[blockIdx.x] = t;
  }
  // the last CTA acknowledges the epoch to every sender (their slots here may be reused), unless some CTA gave up
  if (grid_done_ok(counter, ok != 0))
    for (int r = 0; r < W; ++r)
      if (r != rank) st_release_sys(reinterpret_cast<long long*>(acks.p[r]) + (int64_t)rank * nb + b, epoch);
}

// Weight broadcast of one bucket: fp32 master segment of this owner -> bf16 at the same offsets in every rank's
// compute-weight buffer (its own included); then flag[rank][b] = epoch at every peer.
// Skipped entirely (no stores, no flags) when the status word already holds an error: the reduction that produced the
// master may not have happened.
__global__ void __launch_bounds__(256) p2p_bcast_bf16_kernel(const float* __restrict__ master, PeerTable w16,
                                                             PeerTable flags, unsigned int* counter, int W, int rank,
                                                             int nb, int b, int64_t off, int64_t n, long long epoch,
                                                             const int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = status_clean(err);
  __syncthreads();
  const int64_t n8 = ok ? n / 8 : 0;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n8; j += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = reinterpret_cast<const float4*>(master + off)[2 * j];
    const float4 c = reinterpret_cast<const float4*>(master + off)[2 * j + 1];
    uint4 v;
    v.x = pack_bf16(a.x, a.y);
    v.y = pack_bf16(a.z, a.w);
    v.z = pack_bf16(c.x, c.y);
    v.w = pack_bf16(c.z, c.w);
    for (int r = 0; r < W; ++r)
      reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(w16.p[r]) + off)[j] = v;
  }
  if (grid_done_ok(counter, ok != 0))
    for (int r = 0; r < W; ++r)
      if (r != rank) st_release_sys(reinterpret_cast<long long*>(flags.p[r]) + (int64_t)rank * nb + b, epoch);
}

// waits (one thread) until flags[r][b] >= epoch for every r != rank and every bucket b in [b0, b1)
__global__ void p2p_wait_kernel(const long long* __restrict__ flags, int W, int rank, int nb, int b0, int b1,
                                long long epoch, unsigned long long budget_ns, int* err) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  for (int b = b0; b < b1; ++b)
    for (int r = 0; r < W; ++r)
      if (r != rank && !wait_flag(flags + (int64_t)r * nb + b, epoch, err, budget_ns)) return;
}

// Fused optimizer apply of one bucket's owned parameters, then the bf16 weights to every rank (the sharded update
// and the weight all-gather in one kernel). One CTA per table entry (a chunk of one parameter):
//   kind 0 (AdamW, decoupled decay):  p *= 1 - lr wd;  m = b1 m + (1 - b1) g;  v = b2 v + (1 - b2) g^2;
//                                     p -= (lr / bc1) m / (sqrt(v) / sqrt(bc2) + eps)
//   kind 1 (Muon unit):               p = p (1 - lr_m wd_m) + coef_scale * O      (O: the Newton-Schulz output, bf16;
//                                     coef_scale = -lr_m * coef of the entry)
// then ema = lerp(ema, p, 1 - decay) when an EMA buffer is given, and bf16(p) into every rank's weights at the same
// offset. Gradients arrive clipped. Reference optimizer: baselines/PixelGen/src/optim/muon.py:64-254 (MuonAdamW);
// torch AdamW for the vectors.
struct ApplyEntry {
  int64_t off;
  int32_t n;
  int32_t kind;
  float coef;
  float pad;
};

struct ApplyScalars {
  float lr_a, wd_a, b1, b2, eps, bc1, rsqrt_bc2;  // AdamW (bias corrections of this step)
  float lr_m, wd_m;                             // Muon
  float ema_keep;                               // EMA decay (used when ema != nullptr)
};

__global__ void __launch_bounds__(256) fused_apply_kernel(const ApplyEntry* __restrict__ tab, int nent, float* p,
                                                          const float* __restrict__ g, float* m1, float* m2,
                                                          const __nv_bfloat16* __restrict__ upd, float* ema,
                                                          PeerTable w16, PeerTable wflags, unsigned int* counter,
                                                          ApplyScalars sc, int W, int rank, int nb, int b,
                                                          long long epoch, const int* err) {
  // with an error on the status word (a reduction that gave up), nothing is updated and no flag is raised
  __shared__ int ok;
  if (threadIdx.x == 0) ok = status_clean(err);
  __syncthreads();
  if (ok && (int)blockIdx.x < nent) {
    const ApplyEntry e = tab[blockIdx.x];
    const float keep_a = 1.f - sc.lr_a * sc.wd_a, keep_m = 1.f - sc.lr_m * sc.wd_m;
    const float step_a = sc.lr_a / sc.bc1, mscale = -sc.lr_m * e.coef;
    for (int i0 = threadIdx.x * 8; i0 < e.n; i0 += blockDim.x * 8) {
      const int cnt = min(8, e.n - i0);
      const int64_t o = e.off + i0;
      float pv[8], nv[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (k >= cnt) {
          nv[k] = 0.f;
          continue;
        }
        pv[k] = p[o + k];
        float x;
        if (e.kind == 0) {
          const float gk = g[o + k];
          const float m = sc.b1 * m1[o + k] + (1.f - sc.b1) * gk;
          const float v = sc.b2 * m2[o + k] + (1.f - sc.b2) * gk * gk;
          m1[o + k] = m;
          m2[o + k] = v;
          x = pv[k] * keep_a - step_a * m / (sqrtf(v) * sc.rsqrt_bc2 + sc.eps);
        } else {
          x = pv[k] * keep_m + mscale * __bfloat162float(upd[o + k]);
        }
        p[o + k] = x;
        if (ema != nullptr) ema[o + k] = x + sc.ema_keep * (ema[o + k] - x);
        nv[k] = x;
      }
      if (cnt == 8 && (o & 7) == 0) {
        uint4 v;
        v.x = pack_bf16(nv[0], nv[1]);
        v.y = pack_bf16(nv[2], nv[3]);
        v.z = pack_bf16(nv[4], nv[5]);
        v.w = pack_bf16(nv[6], nv[7]);
        for (int r = 0; r < W; ++r) *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(w16.p[r]) + o) = v;
      } else {
        for (int r = 0; r < W; ++r)
          for (int k = 0; k < cnt; ++k) reinterpret_cast<__nv_bfloat16*>(w16.p[r])[o + k] = __float2bfloat16_rn(nv[k]);
      }
    }
  }
  if (grid_done_ok(counter, ok != 0))
    for (int r = 0; r < W; ++r)
      if (r != rank) st_release_sys(reinterpret_cast<long long*>(wflags.p[r]) + (int64_t)rank * nb + b, epoch);
}

// ------------------------------------------------------------------------------------------------------ host
static void deleter(void* p) { cudaFree(p); }

at::Tensor p2p_alloc(int64_t nbytes, int64_t device) {
  const at::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  void* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, (size_t)nbytes) == cudaSuccess, "p2p_alloc: cudaMalloc failed");
  TORCH_CHECK(cudaMemset(p, 0, (size_t)nbytes) == cudaSuccess, "p2p_alloc: cudaMemset failed");
  return torch::from_blob(p, {nbytes}, deleter, at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device));
}

at::Tensor p2p_export(const at::Tensor& t) {
  cudaIpcMemHandle_t h;
  TORCH_CHECK(cudaIpcGetMemHandle(&h, t.data_ptr()) == cudaSuccess, "cudaIpcGetMemHandle failed");
  at::Tensor out = at::empty({(int64_t)sizeof(h)}, at::TensorOptions().dtype(at::kByte));
  memcpy(out.data_ptr(), &h, sizeof(h));
  return out;
}

int64_t p2p_import(const at::Tensor& handle, int64_t device) {
  const at::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  cudaIpcMemHandle_t h;
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(h), "p2p_import: bad handle");
  memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  TORCH_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess,
              "cudaIpcOpenMemHandle failed (peer access between these GPUs?)");
  return reinterpret_cast<int64_t>(p);
}

void p2p_close(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }

static PeerTable table(const std::vector<int64_t>& v) {
  TORCH_CHECK(v.size() <= 8, "at most 8 ranks");
  PeerTable t{};
  for (size_t i = 0; i < v.size(); ++i) t.p[i] = v[i];
  return t;
}

static int grid_for(int64_t n_vec, int device) {
  static int sms = 0;
  if (sms == 0) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  return (int)std::max<int64_t>(1, std::min<int64_t>((n_vec + 255) / 256, 2 * sms));
}

// push + reduce of bucket b (grad, recv: local fp32 flat buffers; flags/acks: local int64 [W][nb] arrays and the
// peers' addresses of the same arrays); sumsq receives one partial per reduce CTA (its length bounds the grid).
void p2p_reduce_scatter(const at::Tensor& grad, const at::Tensor& recv, const std::vector<int64_t>& peer_recv,
                        const at::Tensor& flags, const std::vector<int64_t>& peer_flags, const at::Tensor& acks,
                        const std::vector<int64_t>& peer_acks, const at::Tensor& counters, const at::Tensor& sumsq,
                        int64_t rank, int64_t nb, int64_t b, int64_t start, int64_t seg, int64_t epoch) {
  const int W = (int)peer_recv.size();
  TORCH_CHECK(seg % 4 == 0 && start % 4 == 0, "p2p_reduce_scatter: 16-byte aligned segments expected");
  const at::cuda::CUDAGuard guard(grad.device());
  auto s = at::cuda::getCurrentCUDAStream();
  unsigned int* ctr = reinterpret_cast<unsigned int*>(counters.data_ptr<int>());
  const int dev = grad.get_device();
  const int gp = grid_for((int64_t)(W - 1) * (seg / 4), dev);
  p2p_push_kernel<<<gp, 256, 0, s>>>(grad.data_ptr<float>(), table(peer_recv), table(peer_flags),
                                     reinterpret_cast<long long*>(acks.data_ptr<int64_t>()), ctr + 2 * b, W, (int)rank,
                                     (int)nb, (int)b, start, seg, (long long)epoch, status_word());
  NG_LAUNCH_CHECK();
  const int gr = std::min<int>(grid_for(seg / 4, dev), (int)sumsq.numel());
  p2p_reduce_kernel<<<gr, 256, 0, s>>>(grad.data_ptr<float>(), recv.data_ptr<float>(),
                                       reinterpret_cast<const long long*>(flags.data_ptr<int64_t>()), table(peer_acks),
                                       ctr + 2 * b + 1, sumsq.data_ptr<float>(), W, (int)rank, (int)nb, (int)b, start,
                                       seg, (long long)epoch, status_word());
  NG_LAUNCH_CHECK();
}

void p2p_bcast_bf16(const at::Tensor& master, const std::vector<int64_t>& peer_w16, const std::vector<int64_t>& peer_flags,
                    const at::Tensor& counters, int64_t rank, int64_t nb, int64_t b, int64_t off, int64_t n,
                    int64_t epoch) {
  const int W = (int)peer_w16.size();
  TORCH_CHECK(n % 8 == 0 && off % 8 == 0, "p2p_bcast_bf16: 16-byte aligned segments expected");
  const at::cuda::CUDAGuard guard(master.device());
  unsigned int* ctr = reinterpret_cast<unsigned int*>(counters.data_ptr<int>());
  p2p_bcast_bf16_kernel<<<grid_for(n / 8, master.get_device()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      master.data_ptr<float>(), table(peer_w16), table(peer_flags), ctr, W, (int)rank, (int)nb, (int)b, off, n,
      (long long)epoch, status_word());
  NG_LAUNCH_CHECK();
}

// table: int64 tensor [nent, 3] on the device (ApplyEntry rows: off | n, kind | coef, pad as raw bits); scalars:
// lr_a, wd_a, b1, b2, eps, bc1, rsqrt_bc2, lr_m, wd_m, ema_keep.
void p2p_fused_apply(const at::Tensor& table_t, int64_t nent, const at::Tensor& p, const at::Tensor& g,
                     const at::Tensor& m1, const at::Tensor& m2, const at::Tensor& upd,
                     const c10::optional<at::Tensor>& ema, const std::vector<int64_t>& peer_w16,
                     const std::vector<int64_t>& peer_wflags, const at::Tensor& counters, std::vector<double> scalars,
                     int64_t rank, int64_t nb, int64_t b, int64_t epoch) {
  static_assert(sizeof(ApplyEntry) == 24, "ApplyEntry layout");
  TORCH_CHECK(scalars.size() == 10, "p2p_fused_apply: 10 scalars");
  TORCH_CHECK(table_t.numel() * 8 >= nent * (int64_t)sizeof(ApplyEntry), "p2p_fused_apply: table too small");
  const at::cuda::CUDAGuard guard(p.device());
  ApplyScalars sc;
  sc.lr_a = (float)scalars[0];
  sc.wd_a = (float)scalars[1];
  sc.b1 = (float)scalars[2];
  sc.b2 = (float)scalars[3];
  sc.eps = (float)scalars[4];
  sc.bc1 = (float)scalars[5];
  sc.rsqrt_bc2 = (float)scalars[6];
  sc.lr_m = (float)scalars[7];
  sc.wd_m = (float)scalars[8];
  sc.ema_keep = (float)scalars[9];
  float* ema_p = (ema.has_value() && ema->defined()) ? ema->data_ptr<float>() : nullptr;
  fused_apply_kernel<<<(unsigned)std::max<int64_t>(1, nent), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const ApplyEntry*>(table_t.data_ptr()), (int)nent, p.data_ptr<float>(), g.data_ptr<float>(),
      m1.data_ptr<float>(), m2.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(upd.data_ptr()), ema_p,
      table(peer_w16), table(peer_wflags), reinterpret_cast<unsigned int*>(counters.data_ptr<int>()), sc,
      (int)peer_w16.size(), (int)rank, (int)nb, (int)b, (long long)epoch, status_word());
  NG_LAUNCH_CHECK();
}

// budget_ns <= 0: the default peer budget (NG_PEER_WAIT_NS)
void p2p_wait(const at::Tensor& flags, int64_t world, int64_t rank, int64_t nb, int64_t b0, int64_t b1,
              int64_t epoch, int64_t budget_ns) {
  const at::cuda::CUDAGuard guard(flags.device());
  p2p_wait_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const long long*>(flags.data_ptr<int64_t>()), (int)world, (int)rank, (int)nb, (int)b0, (int)b1,
      (long long)epoch, budget_ns > 0 ? (unsigned long long)budget_ns : NG_PEER_WAIT_NS, status_word());
  NG_LAUNCH_CHECK();
}

}  // namespace ng
