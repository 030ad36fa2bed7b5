#pragma once
#include <stdint.h>

namespace at {
class Tensor;
}

namespace ng {
// Per-device error word (cudaMalloc'd once per device on first use); 0 = no error.
int* status_word();
int64_t status_read();
void status_clear();
void status_copy_async(const at::Tensor& out);
// Host-side count of kernel launches issued by this extension (the benchmark's launch claim).
void note_launch();
int64_t launch_count();
}  // namespace ng

#include <c10/cuda/CUDAException.h>
// Checks the launch just issued and counts it.
#define NG_LAUNCH_CHECK()            \
  do {                               \
    C10_CUDA_KERNEL_LAUNCH_CHECK();  \
    ::ng::note_launch();             \
  } while (0)
namespace ng {
}  // namespace ng
