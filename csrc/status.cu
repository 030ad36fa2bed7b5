// Device status word shared by every kernel of the extension: kernels that give up a bounded wait (a lost mbarrier
// arrival, a peer flag that never came) write an error code here and return instead of hanging. The host reads and
// clears it between steps (nano_gpic_b200.ops.status).
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "status.h"

namespace ng {

static std::mutex g_mu;
static std::vector<int*> g_words;

int* status_word() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if ((int)g_words.size() <= dev) g_words.resize(dev + 1, nullptr);
  if (g_words[dev] == nullptr) {
    int* p = nullptr;
    TORCH_CHECK(cudaMalloc(&p, sizeof(int)) == cudaSuccess, "status word allocation failed");
    TORCH_CHECK(cudaMemset(p, 0, sizeof(int)) == cudaSuccess, "status word reset failed");
    g_words[dev] = p;
  }
  return g_words[dev];
}

int64_t status_read() {
  int v = 0;
  auto stream = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(cudaMemcpyAsync(&v, status_word(), sizeof(int), cudaMemcpyDeviceToHost, stream) == cudaSuccess);
  TORCH_CHECK(cudaStreamSynchronize(stream) == cudaSuccess);
  return v;
}

static std::atomic<int64_t> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
int64_t launch_count() { return g_launches.load(std::memory_order_relaxed); }

// Enqueues a copy of the word into `out` (a pinned int32 host tensor of one element) on the current stream, without
// waiting: the host reads it later, after an event recorded behind the copy has completed.
void status_copy_async(const at::Tensor& out) {
  TORCH_CHECK(out.device().is_cpu() && out.scalar_type() == at::kInt && out.numel() == 1 && out.is_pinned(),
              "status_copy_async: a pinned int32 host tensor of one element");
  auto stream = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(cudaMemcpyAsync(out.data_ptr<int>(), status_word(), sizeof(int), cudaMemcpyDeviceToHost, stream) ==
              cudaSuccess);
}

void status_clear() {
  auto stream = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(cudaMemsetAsync(status_word(), 0, sizeof(int), stream) == cudaSuccess);
}

}  // namespace ng
