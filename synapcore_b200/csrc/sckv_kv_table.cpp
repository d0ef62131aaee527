// Host-side KV prefix hash table over caller memory.
//
// Slot layout (80 bytes, packed, little-endian) is the reference's
// NativeKVPrefixSlot (native/synapcore_native.mm:93-100):
//   [0,32) prefix_hash  [32,64) parent_hash  [64,68) occupied u32
//   [68,72) token_end u32  [72,80) created_at f64
// Home slot = u32le(prefix_hash[0:4]) & 1023; 64 linear probes.
// Lookup semantics: synapcore_native_kv_lookup (:716-734).
// Insert semantics: synapcore_native_kv_insert (:736-780) — first empty or
// equal slot in the window is (over)written; otherwise the slot with the
// smallest created_at in the window (first such on ties, home slot if none is
// below +inf) is overwritten and its hash reported; when none was below +inf
// the return code is 3 instead of 2, because the reference's Python bridge
// (native/native_engine.py:1747-1752) reports no hash for that case.
#include <cstdint>
#include <cstring>
#include <limits>

#include "sckv.h"

namespace {

constexpr uint32_t kSlots = 1024;
constexpr uint32_t kProbes = 64;
constexpr size_t kSlotBytes = 80;

inline uint32_t home_slot(const uint8_t* h) {
  uint32_t v;
  std::memcpy(&v, h, 4);
  return v & (kSlots - 1);
}

inline uint8_t* slot_ptr(uint8_t* table, uint32_t idx) { return table + static_cast<size_t>(idx) * kSlotBytes; }
inline const uint8_t* slot_ptr(const uint8_t* table, uint32_t idx) {
  return table + static_cast<size_t>(idx) * kSlotBytes;
}

inline uint32_t rd_u32(const uint8_t* p) {
  uint32_t v;
  std::memcpy(&v, p, 4);
  return v;
}
inline double rd_f64(const uint8_t* p) {
  double v;
  std::memcpy(&v, p, 8);
  return v;
}

void write_slot(uint8_t* s, const uint8_t* prefix, const uint8_t* parent, uint32_t token_end, double ts) {
  std::memcpy(s, prefix, 32);
  std::memcpy(s + 32, parent, 32);
  const uint32_t occ = 1u;
  std::memcpy(s + 64, &occ, 4);
  std::memcpy(s + 68, &token_end, 4);
  std::memcpy(s + 72, &ts, 8);
}

}  // namespace

extern "C" int sckv_kv_lookup(const uint8_t* table, const uint8_t* prefix_hash32, uint32_t* out_token_end) {
  if (table == nullptr || prefix_hash32 == nullptr) return 0;
  const uint32_t slot = home_slot(prefix_hash32);
  for (uint32_t probe = 0; probe < kProbes; ++probe) {
    const uint8_t* s = slot_ptr(table, (slot + probe) & (kSlots - 1));
    if (rd_u32(s + 64) == 0u) return 0;
    if (std::memcmp(s, prefix_hash32, 32) == 0) {
      if (out_token_end) *out_token_end = rd_u32(s + 68);
      return 1;
    }
  }
  return 0;
}

extern "C" int sckv_kv_insert(uint8_t* table, const uint8_t* prefix_hash32, const uint8_t* parent_hash32,
                              uint32_t token_end, double timestamp, uint8_t* out_evicted_hash32,
                              uint64_t* evictions) {
  if (table == nullptr || prefix_hash32 == nullptr || parent_hash32 == nullptr) return SCKV_ERR_INVALID_ARG;
  const uint32_t slot = home_slot(prefix_hash32);
  uint32_t oldest = slot;
  double oldest_ts = std::numeric_limits<double>::infinity();
  bool found_older = false;  // some slot had created_at < +inf
  for (uint32_t probe = 0; probe < kProbes; ++probe) {
    const uint32_t idx = (slot + probe) & (kSlots - 1);
    uint8_t* s = slot_ptr(table, idx);
    if (rd_u32(s + 64) == 0u || std::memcmp(s, prefix_hash32, 32) == 0) {
      write_slot(s, prefix_hash32, parent_hash32, token_end, timestamp);
      return 1;
    }
    const double ts = rd_f64(s + 72);
    if (ts < oldest_ts) {
      oldest_ts = ts;
      oldest = idx;
      found_older = true;
    }
  }
  uint8_t* victim = slot_ptr(table, oldest);
  if (out_evicted_hash32) std::memcpy(out_evicted_hash32, victim, 32);
  write_slot(victim, prefix_hash32, parent_hash32, token_end, timestamp);
  if (evictions) ++*evictions;
  // No comparable timestamp in the window: the home slot is overwritten
  // either way; the Python bridge then reports no evicted hash.
  return found_older ? 2 : 3;
}
