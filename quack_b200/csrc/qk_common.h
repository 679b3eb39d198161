// Host-side helpers shared by the translation units of the library.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cstddef>

#include "qk_types.h"

// Records `msg` as the calling thread's last error and returns `code`.
int qk_fail(int code, const char* fmt, ...);
// cudaGetLastError() -> QK_OK or QK_ERR_CUDA (with the CUDA error string recorded).
int qk_check_launch(const char* what);
void qk_count_launch();
