// Host-side declarations of the paged-cache kernels (decode.cu).
#pragma once
#include "common.cuh"

namespace screen {
void kv_append(const screen_kv_append_args& a, cudaStream_t s);
void decode(const screen_decode_args& a, float* part, cudaStream_t s);
int decode_device_status(bool clear);
int xent_device_status(bool clear);
}  // namespace screen
