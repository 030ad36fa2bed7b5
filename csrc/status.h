#pragma once
#include <stdint.h>

namespace ng {
// Per-device error word (cudaMalloc'd once per device on first use); 0 = no error.
int* status_word();
int64_t status_read();
void status_clear();
}  // namespace ng
