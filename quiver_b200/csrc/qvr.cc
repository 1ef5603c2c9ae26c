#include "qvr.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <system_error>

#include "qv_internal.cuh"

namespace qv {
namespace {

constexpr char kMagic[8] = {'Q', 'U', 'I', 'V', 'E', 'R', 'D', 'B'};
constexpr uint32_t kVersion = 1;
constexpr uint32_t kEndian = 0x01020304u;
constexpr size_t kAlign = 64;
constexpr size_t kMaxSections = 64;

struct Header {
  char magic[8];
  uint32_t version, kind, endian_tag, num_sections;
  uint64_t file_size;
  uint32_t table_crc, header_crc;
  uint8_t reserved[24];
};
static_assert(sizeof(Header) == 64, "header layout");
struct Entry {
  uint32_t tag, crc;
  uint64_t offset, size;
};
static_assert(sizeof(Entry) == 24, "entry layout");
constexpr size_t kHeaderCrcSpan = offsetof(Header, header_crc);

size_t align_up(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

std::string errno_text() { return std::generic_category().message(errno); }

// Castagnoli polynomial, reflected (0x82F63B78); byte-at-a-time table.
struct CrcTable {
  uint32_t t[256];
  CrcTable() {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c & 1) ? (c >> 1) ^ 0x82F63B78u : c >> 1;
      t[i] = c;
    }
  }
};

void write_all(int fd, const void* data, size_t size, size_t offset, const std::string& path) {
  const auto* p = static_cast<const char*>(data);
  while (size > 0) {
    const ssize_t n = ::pwrite(fd, p, size, static_cast<off_t>(offset));
    if (n < 0 && errno == EINTR) continue;
    if (n <= 0) fail(QV_ERR_IO, "write to '" + path + "' failed: " + errno_text());
    p += n;
    size -= static_cast<size_t>(n);
    offset += static_cast<size_t>(n);
  }
}

}  // namespace

uint32_t crc32c(const void* data, size_t size, uint32_t crc) {
  static const CrcTable table;
  const auto* p = static_cast<const unsigned char*>(data);
  uint32_t c = ~crc;
  for (size_t i = 0; i < size; ++i) c = table.t[(c ^ p[i]) & 0xff] ^ (c >> 8);
  return ~c;
}

std::string QvrFile::tag_name(uint32_t tag) {
  std::string s(4, '?');
  for (int i = 0; i < 4; ++i) {
    const char c = static_cast<char>((tag >> (8 * i)) & 0xff);
    s[i] = (c >= 32 && c < 127) ? c : '?';
  }
  return "'" + s + "'";
}

void QvrWriter::add(uint32_t tag, const void* data, size_t size) {
  for (const auto& s : sections_)
    if (s.tag == tag) fail(QV_ERR_INVALID, "duplicate section " + QvrFile::tag_name(tag));
  if (sections_.size() >= kMaxSections) fail(QV_ERR_INVALID, "too many sections");
  sections_.push_back({tag, data, size});
}

void QvrWriter::commit(const std::string& path) const {
  static std::atomic<uint64_t> counter{0};
  const std::string tmp = path + ".tmp." + std::to_string(::getpid()) + "." +
                          std::to_string(counter.fetch_add(1));
  const int fd = ::open(tmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
  if (fd < 0) fail(QV_ERR_IO, "cannot create '" + tmp + "': " + errno_text());
  bool ok = false;
  struct Cleanup {
    int fd;
    const std::string& tmp;
    bool& ok;
    ~Cleanup() {
      if (fd >= 0) ::close(fd);
      if (!ok) ::unlink(tmp.c_str());
    }
  } cleanup{fd, tmp, ok};

  std::vector<Entry> table(sections_.size());
  size_t offset = align_up(sizeof(Header) + table.size() * sizeof(Entry));
  for (size_t i = 0; i < sections_.size(); ++i) {
    const Section& s = sections_[i];
    if (s.size > 0) write_all(fd, s.data, s.size, offset, tmp);
    table[i] = Entry{s.tag, crc32c(s.data, s.size), offset, s.size};
    offset = align_up(offset + s.size);
  }
  Header h{};
  std::memcpy(h.magic, kMagic, sizeof(kMagic));
  h.version = kVersion;
  h.kind = static_cast<uint32_t>(kind_);
  h.endian_tag = kEndian;
  h.num_sections = static_cast<uint32_t>(table.size());
  h.file_size = offset;
  h.table_crc = crc32c(table.data(), table.size() * sizeof(Entry));
  h.header_crc = crc32c(&h, kHeaderCrcSpan);
  write_all(fd, table.data(), table.size() * sizeof(Entry), sizeof(Header), tmp);
  write_all(fd, &h, sizeof(h), 0, tmp);
  if (::ftruncate(fd, static_cast<off_t>(offset)) != 0)
    fail(QV_ERR_IO, "resize '" + tmp + "' failed: " + errno_text());
  if (::fsync(fd) != 0) fail(QV_ERR_IO, "fsync '" + tmp + "' failed: " + errno_text());
  if (std::rename(tmp.c_str(), path.c_str()) != 0)
    fail(QV_ERR_IO, "rename to '" + path + "' failed: " + errno_text());
  ok = true;
}

QvrFile::QvrFile(const std::string& path, QvrKind kind, bool verify_checksums) {
  const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) fail(QV_ERR_IO, "cannot open '" + path + "': " + errno_text());
  struct Closer {
    int fd;
    ~Closer() { ::close(fd); }
  } closer{fd};
  struct stat st {};
  if (::fstat(fd, &st) != 0) fail(QV_ERR_IO, "cannot stat '" + path + "': " + errno_text());
  if (!S_ISREG(st.st_mode)) fail(QV_ERR_IO, "'" + path + "' is not a regular file");
  const size_t size = static_cast<size_t>(st.st_size);
  if (size < sizeof(Header)) fail(QV_ERR_IO, "'" + path + "' is too small to be a Quiver index");
  data_.resize(size);
  size_t done = 0;
  while (done < size) {
    const ssize_t n = ::pread(fd, data_.data() + done, size - done, static_cast<off_t>(done));
    if (n < 0 && errno == EINTR) continue;
    if (n <= 0)
      fail(QV_ERR_IO, "read '" + path + "' failed: " + (n == 0 ? "unexpected EOF" : errno_text()));
    done += static_cast<size_t>(n);
  }
  const std::string corrupt = "corrupt index file '" + path + "': ";
  Header h;
  std::memcpy(&h, data_.data(), sizeof(h));
  if (std::memcmp(h.magic, kMagic, sizeof(kMagic)) != 0)
    fail(QV_ERR_IO, "'" + path + "' is not a Quiver index (bad magic)");
  if (h.endian_tag != kEndian)
    fail(QV_ERR_IO, corrupt + "written on a machine with different endianness");
  if (h.header_crc != crc32c(&h, kHeaderCrcSpan)) fail(QV_ERR_IO, corrupt + "header checksum mismatch");
  if (h.version != kVersion)
    fail(QV_ERR_IO, "'" + path + "' uses format version " + std::to_string(h.version) +
                        "; this build reads version " + std::to_string(kVersion));
  if (h.kind != static_cast<uint32_t>(kind))
    fail(QV_ERR_IO, "'" + path + "' holds a different index type");
  if (h.file_size != size)
    fail(QV_ERR_IO, corrupt + "truncated or padded (size " + std::to_string(size) +
                        ", header says " + std::to_string(h.file_size) + ")");
  if (h.num_sections > kMaxSections) fail(QV_ERR_IO, corrupt + "too many sections");
  const size_t table_bytes = h.num_sections * sizeof(Entry);
  if (sizeof(Header) + table_bytes > size) fail(QV_ERR_IO, corrupt + "section table out of bounds");
  if (h.table_crc != crc32c(data_.data() + sizeof(Header), table_bytes))
    fail(QV_ERR_IO, corrupt + "section table checksum mismatch");
  std::vector<Entry> entries(h.num_sections);
  std::memcpy(entries.data(), data_.data() + sizeof(Header), table_bytes);
  const size_t data_start = sizeof(Header) + table_bytes;
  for (const Entry& e : entries) {
    const std::string name = tag_name(e.tag);
    if (e.offset % kAlign != 0) fail(QV_ERR_IO, corrupt + "misaligned section " + name);
    if (e.offset < data_start || e.offset > size || e.size > size - e.offset)
      fail(QV_ERR_IO, corrupt + "section " + name + " out of bounds");
    if (sections_.count(e.tag)) fail(QV_ERR_IO, corrupt + "duplicate section " + name);
    if (verify_checksums && crc32c(data_.data() + e.offset, e.size) != e.crc)
      fail(QV_ERR_IO, corrupt + "checksum mismatch in section " + name);
    sections_[e.tag] = {e.offset, e.size};
  }
  std::sort(entries.begin(), entries.end(),
            [](const Entry& a, const Entry& b) { return a.offset < b.offset; });
  for (size_t i = 1; i < entries.size(); ++i)
    if (entries[i - 1].offset + entries[i - 1].size > entries[i].offset)
      fail(QV_ERR_IO, corrupt + "overlapping sections");
}

const uint8_t* QvrFile::bytes(uint32_t tag, size_t* size) const {
  auto it = sections_.find(tag);
  if (it == sections_.end())
    fail(QV_ERR_IO, "corrupt index file: missing section " + tag_name(tag));
  *size = static_cast<size_t>(it->second.second);
  return data_.data() + it->second.first;
}

const uint8_t* QvrFile::array(uint32_t tag, size_t count, size_t elem) const {
  size_t size = 0;
  const uint8_t* p = bytes(tag, &size);
  if (count > size / elem || size != count * elem)
    fail(QV_ERR_IO, "corrupt index file: section " + tag_name(tag) + " has the wrong size");
  return p;
}

}  // namespace qv
