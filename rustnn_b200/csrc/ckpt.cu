// Checkpoint files in the reference's format (ckpt.rs:8-247): a 27-byte
// header — the magic "RUSTNN\0", the tensor count (u32), the scalar count
// (u64) and the FNV-1a hash of the model configuration (u64), little endian
// — then every parameter tensor in for_each_param order and every buffer in
// for_each_buffer order as little-endian f32.  A save writes `path.tmp` and
// renames it over `path`, so a failed save leaves the previous file alone;
// a load checks the header against the model (or accepts a legacy file that
// is the bare payload) before anything reaches the device.
//
// The optimiser state, which the reference's format leaves out, goes to a
// second file of the same format under the hash of "<kind>-optim".
#include <errno.h>
#include <stdio.h>
#include <string.h>
#include <unistd.h>

#include <string>
#include <vector>

#include "ckpt.cuh"

namespace rnn {

namespace {

constexpr char MAGIC[7] = {'R', 'U', 'S', 'T', 'N', 'N', '\0'};
constexpr size_t HEADER = sizeof(MAGIC) + 4 + 8 + 8;

void put_le(std::vector<uint8_t>& b, uint64_t v, int bytes) {
  for (int i = 0; i < bytes; i++) b.push_back((uint8_t)(v >> (8 * i)));
}

uint64_t get_le(const uint8_t* p, int bytes) {
  uint64_t v = 0;
  for (int i = 0; i < bytes; i++) v |= (uint64_t)p[i] << (8 * i);
  return v;
}

// Little-endian f32 bytes of `n` values (the host is little endian: x86-64
// and aarch64 both; checked at compile time below).
static_assert(__BYTE_ORDER__ == __ORDER_LITTLE_ENDIAN__, "checkpoints are little endian");

}  // namespace

uint64_t ckpt_hash(const char* kind, size_t kind_len, const uint64_t* values, size_t n) {
  // ckpt.rs:83-96: FNV-1a over the kind's bytes, then each value's 8
  // little-endian bytes
  uint64_t h = 0xcbf29ce484222325ULL;
  for (size_t i = 0; i < kind_len; i++) {
    h ^= (uint8_t)kind[i];
    h *= 0x00000100000001b3ULL;
  }
  for (size_t j = 0; j < n; j++)
    for (int i = 0; i < 8; i++) {
      h ^= (uint8_t)(values[j] >> (8 * i));
      h *= 0x00000100000001b3ULL;
    }
  return h;
}

int ckpt_write(const char* path, uint32_t tensors, uint64_t hash, const std::vector<HostPart>& parts) {
  // ckpt.rs:99-128
  RNN_REQUIRE(path && *path, "checkpoint: empty path");
  uint64_t scalars = 0;
  for (const auto& p : parts) scalars += p.len;
  std::vector<uint8_t> head(MAGIC, MAGIC + sizeof(MAGIC));
  put_le(head, tensors, 4);
  put_le(head, scalars, 8);
  put_le(head, hash, 8);
  const std::string tmp = std::string(path) + ".tmp";
  FILE* f = fopen(tmp.c_str(), "wb");
  if (!f) return set_error(RNN_ERR_IO, "checkpoint: cannot create %s: %s", tmp.c_str(), strerror(errno));
  bool ok = fwrite(head.data(), 1, head.size(), f) == head.size();
  for (const auto& p : parts)
    if (ok && p.len) ok = fwrite(p.data, sizeof(float), p.len, f) == p.len;
  ok = ok && fflush(f) == 0 && fsync(fileno(f)) == 0;
  const int err = errno;
  ok = (fclose(f) == 0) && ok;
  if (!ok) {
    remove(tmp.c_str());
    return set_error(RNN_ERR_IO, "checkpoint: writing %s failed: %s", tmp.c_str(), strerror(err));
  }
  if (rename(tmp.c_str(), path) != 0) {
    const int e = errno;
    remove(tmp.c_str());
    return set_error(RNN_ERR_IO, "checkpoint: cannot rename %s to %s: %s", tmp.c_str(), path, strerror(e));
  }
  return RNN_OK;
}

int ckpt_read(const char* path, uint32_t tensors, uint64_t hash, uint64_t scalars, std::vector<float>& payload) {
  // ckpt.rs:130-189
  RNN_REQUIRE(path && *path, "checkpoint: empty path");
  FILE* f = fopen(path, "rb");
  if (!f) return set_error(RNN_ERR_IO, "checkpoint: cannot open %s: %s", path, strerror(errno));
  std::vector<uint8_t> bytes;
  uint8_t buf[1 << 16];
  size_t got;
  while ((got = fread(buf, 1, sizeof(buf), f)) > 0) bytes.insert(bytes.end(), buf, buf + got);
  const bool rerr = ferror(f) != 0;
  fclose(f);
  if (rerr) return set_error(RNN_ERR_IO, "checkpoint: reading %s failed", path);
  const uint64_t expected = scalars * sizeof(float);
  const uint8_t* data = nullptr;
  if (bytes.size() >= sizeof(MAGIC) && memcmp(bytes.data(), MAGIC, sizeof(MAGIC)) == 0) {
    RNN_REQUIRE(bytes.size() >= HEADER, "checkpoint %s: truncated inside the header", path);
    const uint32_t t = (uint32_t)get_le(bytes.data() + 7, 4);
    const uint64_t s = get_le(bytes.data() + 11, 8);
    const uint64_t h = get_le(bytes.data() + 19, 8);
    RNN_REQUIRE(t == tensors, "checkpoint %s has %u tensors; the model expects %u", path, t, tensors);
    RNN_REQUIRE(s == scalars, "checkpoint %s has %llu scalars; the model expects %llu", path,
                (unsigned long long)s, (unsigned long long)scalars);
    RNN_REQUIRE(h == hash, "checkpoint %s is incompatible with the configuration (hash %016llx, expected %016llx)",
                path, (unsigned long long)h, (unsigned long long)hash);
    RNN_REQUIRE(bytes.size() - HEADER == expected, "checkpoint %s: payload has %zu bytes; expected %llu", path,
                bytes.size() - HEADER, (unsigned long long)expected);
    data = bytes.data() + HEADER;
  } else if (bytes.size() == expected) {
    fprintf(stderr, "warning: legacy checkpoint without a header: %s\n", path);
    data = bytes.data();
  } else {
    return set_error(RNN_ERR_ARG, "checkpoint %s: no magic and not a legacy payload (%zu bytes; expected %llu)", path,
                     bytes.size(), (unsigned long long)expected);
  }
  payload.resize(scalars);
  if (scalars) memcpy(payload.data(), data, expected);
  return RNN_OK;
}

}  // namespace rnn

extern "C" uint64_t rnn_ckpt_config_hash(const char* kind, size_t kind_len, const uint64_t* values, size_t n) {
  return rnn::ckpt_hash(kind, kind_len, values, n);
}

extern "C" int rnn_ckpt_write(const char* path, uint32_t tensors, uint64_t config_hash, const float* payload,
                              size_t scalars) {
  RNN_REQUIRE(payload || scalars == 0, "checkpoint: null payload");
  return rnn::ckpt_write(path, tensors, config_hash, {{payload, scalars}});
}

extern "C" int rnn_ckpt_read(const char* path, uint32_t tensors, uint64_t config_hash, float* payload,
                             size_t scalars) {
  RNN_REQUIRE(payload || scalars == 0, "checkpoint: null payload");
  std::vector<float> v;
  RNN_TRY(rnn::ckpt_read(path, tensors, config_hash, scalars, v));
  if (scalars) memcpy(payload, v.data(), scalars * sizeof(float));
  return RNN_OK;
}
