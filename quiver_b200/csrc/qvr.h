// Reader and writer for Quiver's .qvr index container, so indexes move between the reference CPU
// library and this GPU library in both directions.
//
// Layout (src/internal/file_format.h:1-58 of the reference): a 64-byte header (magic "QUIVERDB",
// version 1, index kind, endian tag 0x01020304, section count, file size, CRC-32C of the section
// table, CRC-32C of the header bytes before that field), then 24-byte section entries (fourcc tag,
// CRC-32C, offset, size), then the sections, each on a 64-byte boundary. All little-endian.
#pragma once

#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace qv {

enum class QvrKind : uint32_t { kFlat = 1, kHnsw = 2, kIvfPq = 3 };

constexpr uint32_t fourcc(const char (&s)[5]) {
  return static_cast<uint32_t>(static_cast<unsigned char>(s[0])) |
         static_cast<uint32_t>(static_cast<unsigned char>(s[1])) << 8 |
         static_cast<uint32_t>(static_cast<unsigned char>(s[2])) << 16 |
         static_cast<uint32_t>(static_cast<unsigned char>(s[3])) << 24;
}

uint32_t crc32c(const void* data, size_t size, uint32_t crc = 0);

// Sections are written in the order added; commit() writes to a temporary file, fsyncs it and
// renames it over `path` so readers never see a partial file.
class QvrWriter {
 public:
  explicit QvrWriter(QvrKind kind) : kind_(kind) {}
  void add(uint32_t tag, const void* data, size_t size);
  void commit(const std::string& path) const;

 private:
  struct Section {
    uint32_t tag;
    const void* data;
    size_t size;
  };
  QvrKind kind_;
  std::vector<Section> sections_;
};

// Reads and validates a whole file: magic, endianness, header and table checksums, version, kind,
// size, section bounds/alignment/duplicates/overlap and (optionally) every section's checksum.
// Throws qv::Failure(QV_ERR_IO) with the reference's message wording on any problem.
class QvrFile {
 public:
  QvrFile(const std::string& path, QvrKind kind, bool verify_checksums);
  bool has(uint32_t tag) const { return sections_.count(tag) != 0; }
  // Bytes of a required section.
  const uint8_t* bytes(uint32_t tag, size_t* size) const;
  // A required section that must hold exactly `count` elements of `elem` bytes.
  const uint8_t* array(uint32_t tag, size_t count, size_t elem) const;
  size_t size() const { return data_.size(); }
  static std::string tag_name(uint32_t tag);

 private:
  std::vector<uint8_t> data_;
  std::map<uint32_t, std::pair<uint64_t, uint64_t>> sections_;  // tag -> (offset, size)
};

}  // namespace qv
