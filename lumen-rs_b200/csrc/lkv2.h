// The LKV2 on-disk snapshot format of crates/lumen-mlx/src/kv_disk.rs
// (layout :285-323, records :155-248, manifest :250-283), host side only:
//
//   [4] "LKV2" | [4] version 2 u32 | [4] manifest JSON length u32 | JSON |
//   [4] CRC-32 of the JSON | [4] record count u32 | records ...
//   record: [1] dtype tag | [4] ndim u32 | [ndim x 4] shape i32 |
//           [8] payload bytes u64 | payload | [4] CRC-32 of the record
//
// All little-endian; the CRC is CRC-32/IEEE (crc32fast); the reader rejects
// a payload length that disagrees with shape x dtype, CRC mismatches and
// trailing bytes, as the reference's reader does.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace lc {

// DtypeTag bytes (kv_disk.rs:85-100).
enum Lkv2Dtype : uint8_t {
  kLkvBool = 0, kLkvU8 = 1, kLkvU16 = 2, kLkvU32 = 3, kLkvU64 = 4, kLkvI8 = 5, kLkvI16 = 6, kLkvI32 = 7,
  kLkvI64 = 8, kLkvF16 = 9, kLkvF32 = 10, kLkvF64 = 11, kLkvBF16 = 12,
};
int lkv2_elem_size(uint8_t dtype);  // -1 for an unknown tag

struct Lkv2Record {
  uint8_t dtype = kLkvU8;
  std::vector<int32_t> shape;
  std::vector<uint8_t> data;
  int64_t elems() const;
};

// LayerMeta (kv_disk.rs:214-248); optional fields are -1 when absent.
struct Lkv2Layer {
  std::string kind;
  uint64_t offset = 0, base_offset = 0;
  std::vector<int64_t> arrays;  // record index per slot, -1 = null
  int64_t lengths_id = -1, left_padding_id = -1;
  int64_t max_size = -1, keep = -1, idx = -1, bits = -1, qjl_m = -1, group_size = -1;
  // Not in the reference's LayerMeta (its readers ignore unknown fields):
  // the V bit width when it differs from `bits`.
  int64_t v_bits = -1;
};

// KvManifest (kv_disk.rs:255-283).
struct Lkv2Manifest {
  std::string model_fingerprint;
  uint64_t created_at_unix = 0;
  uint64_t position = 0;
  std::vector<uint32_t> prefix_tokens;
  int64_t last_token = -1;
  bool is_deep = false;
  std::vector<Lkv2Layer> layers;
};

uint32_t crc32_ieee(const uint8_t* p, size_t n, uint32_t crc = 0);

// serde_json's compact form of the manifest, fields in declaration order,
// `skip_serializing_if = "Option::is_none"` fields left out when absent.
std::string lkv2_manifest_json(const Lkv2Manifest& m);
// Parses a manifest (any field order, unknown fields ignored); throws
// Error(LC_ERR_IO) on malformed JSON.
Lkv2Manifest lkv2_parse_manifest(const std::string& json);

// Throw Error: LC_ERR_IO (open/read/write failure, CRC, truncation,
// trailing bytes, inconsistent lengths), LC_ERR_MAGIC (magic or version).
void lkv2_write(const std::string& path, const Lkv2Manifest& m, const std::vector<Lkv2Record>& recs);
void lkv2_read(const std::string& path, Lkv2Manifest& m, std::vector<Lkv2Record>& recs);

}  // namespace lc
