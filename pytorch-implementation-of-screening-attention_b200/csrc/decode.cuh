// Host-side declarations of the paged-cache kernels (decode.cu).
#pragma once
#include "common.cuh"

namespace screen {
void kv_append(const screen_kv_append_args& a, cudaStream_t s);
void decode(const screen_decode_args& a, float* part, cudaStream_t s);
// append the one new k / v row per (b, h) of ap, then decode, in one launch
// where the bulk-copy kernel serves the cache
void decode_append(const screen_kv_append_args& ap, const screen_decode_args& a, float* part,
                   cudaStream_t s);
int decode_device_status(bool clear);
int xent_device_status(bool clear);
}  // namespace screen
