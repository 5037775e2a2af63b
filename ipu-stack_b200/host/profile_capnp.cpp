// Profile reports in the reference's Cap'n Proto format (include/ipug.h).
//
// The reference writes its cycle profile with the capnp crate
// (ProfileReport::write, crates/ipu-package/src/lib.rs:198-222) against
// schemas/profile.capnp and schemas/profile_common.capnp.  No Cap'n Proto
// library is part of this build, so the message is laid out here directly
// from the published encoding: one segment of 64-bit words, struct pointers
// (tag 0) and list pointers (tag 1) with word offsets relative to the end of
// the pointer, composite lists with a tag word, Text as a NUL-terminated byte
// list, and the stream framing of capnp::serialize (segment count - 1, then
// each segment's size in words, padded to 8 bytes).
//
// Field placement follows the capnp layout rule (fields in ordinal order,
// each taking the first free hole of its size, else splitting a larger hole,
// else a new data word):
//   Profile          data 2 words, 1 pointer: schemaVersion u32 @byte 0,
//                    clockHz u64 @byte 8; tiles -> ptr 0
//   TileProfile      data 1, ptrs 1: physicalTile u32 @0; samples -> ptr 0
//   CycleSample      data 1, ptrs 1: startCycle u32 @0, endCycle u32 @4;
//                    step -> ptr 0
//   Step             data 3, ptrs 4: localIndex u32 @0, phase u32 @4,
//                    epoch u32 @8, kind u16 @12, exchangeEventCycles u32 @16;
//                    operation, kernel, metadata, exchangeActivities -> ptrs 0-3
//   Metadata         data 0, ptrs 2: name, value
//   ExchangeActivity data 2, ptrs 0: kind u16 @0, startCycle u32 @4,
//                    endCycle u32 @8
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/ipug.h"

namespace ipuc {
ipuc_status fail(ipuc_status st, const std::string &msg);
}  // namespace ipuc

namespace ipug_capnp {

// List pointers carry element and word counts in 29 bits; larger lists or
// texts make the builder fail instead of wrapping.
constexpr uint64_t kMaxListCount = (1ull << 29) - 1;

class Builder {
 public:
  bool overflow = false;
  // Allocate n zeroed words; returns the index of the first.
  uint32_t alloc(uint32_t n) {
    const uint32_t at = static_cast<uint32_t>(w_.size());
    w_.resize(w_.size() + n, 0);
    return at;
  }
  void put32(uint32_t word, uint32_t byte, uint32_t v) { std::memcpy(bytes(word) + byte, &v, 4); }
  void put16(uint32_t word, uint32_t byte, uint16_t v) { std::memcpy(bytes(word) + byte, &v, 2); }
  void put64(uint32_t word, uint32_t byte, uint64_t v) { std::memcpy(bytes(word) + byte, &v, 8); }

  // Struct pointer at word `ptr` to a struct whose data section starts at `target`.
  void struct_ptr(uint32_t ptr, uint32_t target, uint16_t data_words, uint16_t ptr_words) {
    const int64_t off = static_cast<int64_t>(target) - (static_cast<int64_t>(ptr) + 1);
    w_[ptr] = (static_cast<uint64_t>(static_cast<uint32_t>(off) << 2)) | (uint64_t(data_words) << 32) |
              (uint64_t(ptr_words) << 48);
  }
  // Allocate a struct and point `ptr` at it; returns the struct's first word.
  uint32_t new_struct(uint32_t ptr, uint16_t data_words, uint16_t ptr_words) {
    const uint32_t at = alloc(data_words + ptr_words);
    struct_ptr(ptr, at, data_words, ptr_words);
    return at;
  }
  // Composite list of n structs at pointer `ptr`; returns the first element's word.
  uint32_t new_struct_list(uint32_t ptr, uint32_t n, uint16_t data_words, uint16_t ptr_words) {
    const uint32_t per = data_words + ptr_words;
    if ((uint64_t)n * per > kMaxListCount || w_.size() + 1 + (uint64_t)n * per > kMaxListCount) {
      overflow = true;
      return alloc(0);
    }
    const uint32_t tag = alloc(1 + n * per);
    w_[tag] = (static_cast<uint64_t>(n) << 2) | (uint64_t(data_words) << 32) | (uint64_t(ptr_words) << 48);
    list_ptr(ptr, tag, 7, n * per);
    return tag + 1;
  }
  // Text (NUL-terminated byte list) at pointer `ptr`.
  void text(uint32_t ptr, const char *s) {
    const size_t len = s ? std::strlen(s) : 0;
    if (len + 1 > kMaxListCount || w_.size() + (len + 8) / 8 > kMaxListCount) {
      overflow = true;
      return;
    }
    const uint32_t at = alloc(static_cast<uint32_t>((len + 1 + 7) / 8));
    if (len) std::memcpy(bytes(at), s, len);
    list_ptr(ptr, at, 2, static_cast<uint32_t>(len + 1));
  }
  // Stream framing of a single segment.
  std::string frame() const {
    std::string out(8 + w_.size() * 8, '\0');
    const uint32_t head[2] = {0u, static_cast<uint32_t>(w_.size())};
    std::memcpy(&out[0], head, 8);
    if (!w_.empty()) std::memcpy(&out[8], w_.data(), w_.size() * 8);
    return out;
  }

 private:
  unsigned char *bytes(uint32_t word) { return reinterpret_cast<unsigned char *>(&w_[word]); }
  void list_ptr(uint32_t ptr, uint32_t target, uint32_t elem_size, uint32_t count) {
    const int64_t off = static_cast<int64_t>(target) - (static_cast<int64_t>(ptr) + 1);
    w_[ptr] = 1u | (static_cast<uint64_t>(static_cast<uint32_t>(off) << 2)) |
              (static_cast<uint64_t>(elem_size) << 32) | (static_cast<uint64_t>(count) << 35);
  }
  std::vector<uint64_t> w_;
};

constexpr uint32_t kSchemaVersion = 5;  // crates/ipu-package/src/lib.rs:201,262

ipuc_status too_large() {
  return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "profile_encode: report larger than a Cap'n Proto segment");
}

ipuc_status encode(uint64_t clock_hz, const ipug_profile_tile *tiles, uint64_t tile_count, std::string &out) {
  if (tile_count && !tiles) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "profile_encode: null tiles");
  if (tile_count > 0x1FFFFFFFu) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "profile_encode: too many tiles");
  Builder b;
  const uint32_t root_ptr = b.alloc(1);
  const uint32_t root = b.new_struct(root_ptr, 2, 1);
  b.put32(root, 0, kSchemaVersion);
  b.put64(root, 8, clock_hz);
  const uint32_t tile0 = b.new_struct_list(root + 2, static_cast<uint32_t>(tile_count), 1, 1);
  if (b.overflow) return too_large();
  for (uint64_t t = 0; t < tile_count; ++t) {
    const ipug_profile_tile &tile = tiles[t];
    if (tile.sample_count && !tile.samples)
      return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "profile_encode: null samples");
    if (tile.sample_count > 0x0FFFFFFFu)
      return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "profile_encode: too many samples");
    const uint32_t tw = tile0 + static_cast<uint32_t>(t) * 2;
    b.put32(tw, 0, tile.physical_tile);
    const uint32_t s0 = b.new_struct_list(tw + 1, static_cast<uint32_t>(tile.sample_count), 1, 1);
    if (b.overflow) return too_large();
    for (uint64_t i = 0; i < tile.sample_count; ++i) {
      const ipug_profile_sample &sm = tile.samples[i];
      if (sm.kind > IPUG_STEP_IDLE) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "profile_encode: step kind out of range");
      if (sm.metadata_count && !sm.metadata)
        return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "profile_encode: null metadata");
      if (sm.activity_count && !sm.activities)
        return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "profile_encode: null activities");
      const uint32_t sw = s0 + static_cast<uint32_t>(i) * 2;
      b.put32(sw, 0, sm.start_cycle);
      b.put32(sw, 4, sm.end_cycle);
      const uint32_t st = b.new_struct(sw + 1, 3, 4);
      b.put32(st, 0, sm.local_index);
      b.put32(st, 4, sm.phase);
      b.put32(st, 8, sm.epoch);
      b.put16(st, 12, static_cast<uint16_t>(sm.kind));
      b.put32(st, 16, sm.exchange_event_cycles);
      b.text(st + 3, sm.operation);
      b.text(st + 4, sm.kernel);
      const uint32_t m0 = b.new_struct_list(st + 5, sm.metadata_count, 0, 2);
      if (b.overflow) return too_large();
      for (uint32_t j = 0; j < sm.metadata_count; ++j) {
        b.text(m0 + 2 * j, sm.metadata[2 * j]);
        b.text(m0 + 2 * j + 1, sm.metadata[2 * j + 1]);
      }
      const uint32_t a0 = b.new_struct_list(st + 6, sm.activity_count, 2, 0);
      if (b.overflow) return too_large();
      for (uint32_t j = 0; j < sm.activity_count; ++j) {
        const ipug_exchange_activity &a = sm.activities[j];
        if (a.kind > 2) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "profile_encode: activity kind out of range");
        b.put16(a0 + 2 * j, 0, static_cast<uint16_t>(a.kind));
        b.put32(a0 + 2 * j, 4, a.start_cycle);
        b.put32(a0 + 2 * j + 1, 0, a.end_cycle);
      }
    }
  }
  if (b.overflow) return too_large();
  out = b.frame();
  return IPUC_OK;
}

ipuc_status deliver(const std::string &bytes, void *buf, uint64_t size, uint64_t *needed, const char *who) {
  if (needed) *needed = bytes.size();
  if (!buf || size < bytes.size())
    return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, std::string(who) + ": buffer too small");
  std::memcpy(buf, bytes.data(), bytes.size());
  return IPUC_OK;
}

}  // namespace ipug_capnp

extern "C" ipuc_status ipug_profile_encode(uint64_t clock_hz, const ipug_profile_tile *tiles, uint64_t tile_count,
                                           void *buf, uint64_t size, uint64_t *needed) {
  std::string bytes;
  const ipuc_status st = ipug_capnp::encode(clock_hz, tiles, tile_count, bytes);
  if (st != IPUC_OK) return st;
  return ipug_capnp::deliver(bytes, buf, size, needed, "profile_encode");
}
