// Checkpoint files in the reference's format (ckpt.rs:8-247); the model
// entry points (resnet.cu, vit.cu) copy their flat device buffers through
// these host routines.
#pragma once

#include <vector>

#include "common.cuh"

namespace rnn {

struct HostPart {
  const float* data;
  size_t len;
};

// FNV-1a of the kind's bytes and each value's 8 little-endian bytes
// (ckpt.rs:83-96).
uint64_t ckpt_hash(const char* kind, size_t kind_len, const uint64_t* values, size_t n);
// Header + the parts' f32 values, written to path.tmp and renamed over path.
int ckpt_write(const char* path, uint32_t tensors, uint64_t hash, const std::vector<HostPart>& parts);
// Validates the header against (tensors, scalars, hash), or accepts a bare
// legacy payload of the expected size; fills `payload` with `scalars` values.
int ckpt_read(const char* path, uint32_t tensors, uint64_t hash, uint64_t scalars, std::vector<float>& payload);

}  // namespace rnn
