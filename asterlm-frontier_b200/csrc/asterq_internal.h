// Internal host/device declarations shared by the asterq translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include "asterq.h"

namespace asterq {

// float32(sqrt(2^k)) for k = 0..10, i.e. the divisor the reference uses in
// normalized_fwht (quantization/kv.py:32: y / math.sqrt(n), a float32 tensor
// divided by a Python float, which torch rounds to float32).
__device__ __constant__ static const float kSqrtTable[11] = {
    1.0f,         1.41421353816986083984375f, 2.0f, 2.8284270763397216796875f, 4.0f, 5.656854152679443359375f,
    8.0f,         11.31370830535888671875f,   16.0f, 22.6274166107177734375f, 32.0f};

int set_error(int status, const char* fmt, ...);
void clear_error();
int check_launch(const char* what);

}  // namespace asterq
