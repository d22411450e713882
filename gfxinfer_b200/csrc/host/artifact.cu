// `.gfxi` v1 artifact container (host code): reader (mmap + validation), streaming
// writer, CRC64-ECMA and their C ABI (include/gfxb/artifact.h).
//
// The byte layout is the reference's (src/artifact.cpp:27-64): fields are
// serialised explicitly, little-endian, at the reference's offsets, so the
// two implementations exchange files. Validation follows ArtifactView::open
// (artifact.cpp:274-407) rule for rule.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <array>
#include <cerrno>
#include <cstring>
#include <limits>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "artifact_internal.h"
#include "kernels/common.cuh"

namespace gfxb::gfxi {
namespace {

constexpr std::array<std::uint8_t, 8> kMagic{'G', 'F', 'X', 'I', '\r', '\n', 0x1a, '\n'};
constexpr std::uint32_t kEndianTag = 0x01020304u;
constexpr std::uint32_t kHeaderBytes = 256;
constexpr std::uint32_t kEntryBytes = 128;

// Header field offsets (artifact.cpp:27-47).
enum : std::size_t {
  kHVersion = 8, kHHeaderBytes = 12, kHEndian = 16, kHFlags = 20, kHDirectory = 24, kHTensorCount = 32,
  kHEntryBytes = 36, kHStringsOffset = 40, kHStringsBytes = 48, kHDataOffset = 56, kHDataBytes = 64,
  kHFileBytes = 72, kHManifestCrc = 80, kHTargetArch = 88, kHModelId = 104, kHWeightsId = 136, kHRecipeId = 168
};
// Directory entry field offsets (artifact.cpp:49-64).
enum : std::size_t {
  kENameOffset = 0, kENameBytes = 8, kEDtype = 12, kEQuant = 14, kERank = 16, kEFlags = 18, kEAlignment = 20,
  kEDims = 24, kEDataOffset = 56, kEDataBytes = 64, kEAuxOffset = 72, kEAuxBytes = 80, kEDataCrc = 88
};

template <class T>
T get(const std::byte* base, std::size_t offset) {
  T value;
  std::memcpy(&value, base + offset, sizeof value);  // the host is little-endian, as the format
  return value;
}
template <class T>
void put(std::byte* base, std::size_t offset, T value) {
  std::memcpy(base + offset, &value, sizeof value);
}

std::uint64_t align_up(std::uint64_t value, std::uint64_t alignment) {
  if (alignment == 0 || (alignment & (alignment - 1)) != 0) return 0;
  if (value > std::numeric_limits<std::uint64_t>::max() - (alignment - 1)) return 0;
  return (value + alignment - 1) & ~(alignment - 1);
}

bool in_file(std::uint64_t offset, std::uint64_t bytes, std::uint64_t file_bytes) {
  return offset <= file_bytes && bytes <= file_bytes - offset;
}

int io_error(const char* action, const std::string& path) {
  const std::string message = std::string(action) + " " + path + ": " + std::strerror(errno);
  return fail(GFXB_IO_ERROR, message.c_str());
}

int corrupt(const std::string& message) { return fail(GFXB_CORRUPT_ARTIFACT, message.c_str()); }

template <std::size_t N>
bool fixed_string(const std::byte* field, char (&out)[N]) {
  std::memcpy(out, field, N);
  const void* end = std::memchr(out, '\0', N);
  if (end == nullptr) return false;  // the identity strings must fit with their terminator here
  return out[0] != '\0';
}

template <std::size_t N>
bool valid_identity_field(const char (&field)[N]) {
  const void* end = std::memchr(field, '\0', N);
  return end != nullptr && field[0] != '\0';
}

int write_at(int fd, const void* source, std::uint64_t bytes, std::uint64_t offset) {
  const auto* cursor = static_cast<const std::byte*>(source);
  while (bytes != 0) {
    const std::size_t chunk = static_cast<std::size_t>(std::min<std::uint64_t>(bytes, 1ull << 30));
    const ssize_t written = ::pwrite(fd, cursor, chunk, static_cast<off_t>(offset));
    if (written < 0) {
      if (errno == EINTR) continue;
      return io_error("write failed for", "artifact");
    }
    if (written == 0) return fail(GFXB_IO_ERROR, "artifact write made no progress");
    cursor += written;
    bytes -= static_cast<std::uint64_t>(written);
    offset += static_cast<std::uint64_t>(written);
  }
  return GFXB_OK;
}

struct Crc64Table {
  std::uint64_t value[256];
  Crc64Table() {
    constexpr std::uint64_t kPolynomial = 0x42F0E1EBA9EA3693ull;  // ECMA-182, MSB first
    for (unsigned byte = 0; byte < 256; ++byte) {
      std::uint64_t crc = static_cast<std::uint64_t>(byte) << 56;
      for (int bit = 0; bit < 8; ++bit) crc = (crc >> 63) != 0 ? (crc << 1) ^ kPolynomial : crc << 1;
      value[byte] = crc;
    }
  }
};

}  // namespace

std::uint64_t crc64(std::uint64_t state, const void* bytes, std::size_t size) noexcept {
  static const Crc64Table table;
  const auto* p = static_cast<const std::uint8_t*>(bytes);
  for (std::size_t i = 0; i < size; ++i) state = table.value[static_cast<std::uint8_t>(state >> 56) ^ p[i]] ^ (state << 8);
  return state;
}

// Tensor names: relative, portable path bytes, no "..".
bool valid_name(const std::string& name) noexcept {
  if (name.empty() || name.front() == '/' || name.find("..") != std::string::npos) return false;
  return std::all_of(name.begin(), name.end(), [](unsigned char c) {
    return (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || (c >= '0' && c <= '9') || c == '_' || c == '-' ||
           c == '.' || c == '/';
  });
}

// ---------------------------------------------------------------------------
// reader
// ---------------------------------------------------------------------------

View::~View() {
  if (mapping_ != nullptr) ::munmap(const_cast<std::byte*>(mapping_), static_cast<std::size_t>(bytes_));
  if (fd_ >= 0) ::close(fd_);
}

const Tensor* View::find(const std::string& name) const {
  const auto it = index_.find(name);
  return it == index_.end() ? nullptr : &tensors_[it->second];
}

void View::fill(const Tensor& t, gfxb_tensor_view& out) const {
  out.name = t.name.c_str();
  out.dtype = t.dtype;
  out.quantization = t.quantization;
  out.rank = t.rank;
  out.flags = t.flags;
  out.alignment = t.alignment;
  for (int i = 0; i < 4; ++i) out.dimensions[i] = t.dimensions[i];
  out.data = data(t);
  out.data_bytes = t.data_bytes;
  out.aux = aux(t);
  out.aux_bytes = t.aux_bytes;
  out.data_offset = t.data_offset;
  out.aux_offset = t.aux_offset;
  out.data_crc64 = t.data_crc64;
}

int View::open(const char* path, bool verify_checksums) {
  fd_ = ::open(path, O_RDONLY | O_CLOEXEC);
  if (fd_ < 0) return io_error("cannot open", path);
  struct stat st {};
  if (::fstat(fd_, &st) != 0) return io_error("cannot stat", path);
  if (st.st_size < static_cast<off_t>(kHeaderBytes)) return corrupt("artifact is smaller than its header");
  bytes_ = static_cast<std::uint64_t>(st.st_size);
  void* mapping = ::mmap(nullptr, static_cast<std::size_t>(bytes_), PROT_READ, MAP_PRIVATE, fd_, 0);
  if (mapping == MAP_FAILED) return io_error("cannot map", path);
  mapping_ = static_cast<const std::byte*>(mapping);
  const std::byte* h = mapping_;

  if (std::memcmp(h, kMagic.data(), kMagic.size()) != 0) return corrupt("invalid .gfxi magic");
  if (get<std::uint32_t>(h, kHVersion) != kVersion || get<std::uint32_t>(h, kHHeaderBytes) != kHeaderBytes) {
    return fail(GFXB_UNSUPPORTED, "unsupported .gfxi artifact version");
  }
  if (get<std::uint32_t>(h, kHEndian) != kEndianTag) return fail(GFXB_UNSUPPORTED, "artifact byte order is unsupported");
  if (get<std::uint32_t>(h, kHEntryBytes) != kEntryBytes) return corrupt("unexpected directory entry size");
  const std::uint64_t file_bytes = get<std::uint64_t>(h, kHFileBytes);
  if (file_bytes != bytes_) return corrupt("artifact length does not match header");
  const std::uint64_t directory_offset = get<std::uint64_t>(h, kHDirectory);
  const std::uint32_t count = get<std::uint32_t>(h, kHTensorCount);
  const std::uint64_t directory_bytes = static_cast<std::uint64_t>(count) * kEntryBytes;
  const std::uint64_t strings_offset = get<std::uint64_t>(h, kHStringsOffset);
  const std::uint64_t strings_bytes = get<std::uint64_t>(h, kHStringsBytes);
  const std::uint64_t data_offset = get<std::uint64_t>(h, kHDataOffset);
  const std::uint64_t data_bytes = get<std::uint64_t>(h, kHDataBytes);
  if (!in_file(directory_offset, directory_bytes, file_bytes) || !in_file(strings_offset, strings_bytes, file_bytes) ||
      !in_file(data_offset, data_bytes, file_bytes) || strings_offset != directory_offset + directory_bytes ||
      data_offset < strings_offset + strings_bytes) {
    return corrupt("artifact section bounds are invalid");
  }
  if (verify_checksums &&
      crc64(0, mapping_ + directory_offset, static_cast<std::size_t>(directory_bytes + strings_bytes)) !=
          get<std::uint64_t>(h, kHManifestCrc)) {
    return corrupt("artifact manifest checksum mismatch");
  }
  if (!fixed_string(h + kHTargetArch, identity_.target_arch) || !fixed_string(h + kHModelId, identity_.model_id) ||
      !fixed_string(h + kHWeightsId, identity_.weights_id) || !fixed_string(h + kHRecipeId, identity_.recipe_id)) {
    return corrupt("artifact identity is incomplete");
  }

  const std::byte* strings = mapping_ + strings_offset;
  std::vector<std::pair<std::uint64_t, std::uint64_t>> ranges;
  tensors_.reserve(count);
  for (std::uint32_t i = 0; i < count; ++i) {
    const std::byte* e = mapping_ + directory_offset + static_cast<std::uint64_t>(i) * kEntryBytes;
    Tensor t;
    const std::uint64_t name_offset = get<std::uint64_t>(e, kENameOffset);
    const std::uint32_t name_bytes = get<std::uint32_t>(e, kENameBytes);
    t.dtype = get<std::uint16_t>(e, kEDtype);
    t.quantization = get<std::uint16_t>(e, kEQuant);
    t.rank = get<std::uint16_t>(e, kERank);
    t.flags = get<std::uint16_t>(e, kEFlags);
    t.alignment = get<std::uint32_t>(e, kEAlignment);
    for (int d = 0; d < 4; ++d) t.dimensions[d] = get<std::uint64_t>(e, kEDims + 8 * d);
    t.data_offset = get<std::uint64_t>(e, kEDataOffset);
    t.data_bytes = get<std::uint64_t>(e, kEDataBytes);
    t.aux_offset = get<std::uint64_t>(e, kEAuxOffset);
    t.aux_bytes = get<std::uint64_t>(e, kEAuxBytes);
    t.data_crc64 = get<std::uint64_t>(e, kEDataCrc);
    if (t.rank > 4 || t.dtype < GFXB_DTYPE_U8 || t.dtype > GFXB_DTYPE_F32 || t.quantization > GFXB_QUANT_FP8_ROW ||
        name_bytes == 0 || !in_file(name_offset, name_bytes, strings_bytes)) {
      return corrupt("invalid tensor directory entry");
    }
    t.name.assign(reinterpret_cast<const char*>(strings + name_offset), name_bytes);
    if (!valid_name(t.name) || index_.count(t.name) != 0) return corrupt("invalid or duplicate tensor name: " + t.name);
    if (t.alignment < kFileAlignment || (t.alignment & (t.alignment - 1)) != 0 || t.data_offset % t.alignment != 0 ||
        !in_file(t.data_offset, t.data_bytes, file_bytes) || t.data_offset < data_offset) {
      return corrupt("invalid tensor payload bounds: " + t.name);
    }
    if (t.aux_bytes != 0 && (t.aux_offset % t.alignment != 0 || !in_file(t.aux_offset, t.aux_bytes, file_bytes) ||
                             t.aux_offset < data_offset)) {
      return corrupt("invalid tensor auxiliary bounds: " + t.name);
    }
    if (verify_checksums && crc64(0, mapping_ + t.data_offset, static_cast<std::size_t>(t.data_bytes)) != t.data_crc64) {
      return corrupt("tensor checksum mismatch: " + t.name);
    }
    ranges.emplace_back(t.data_offset, t.data_offset + t.data_bytes);
    if (t.aux_bytes != 0) ranges.emplace_back(t.aux_offset, t.aux_offset + t.aux_bytes);
    index_.emplace(t.name, tensors_.size());
    tensors_.push_back(std::move(t));
  }
  std::sort(ranges.begin(), ranges.end());
  for (std::size_t i = 1; i < ranges.size(); ++i) {
    if (ranges[i].first < ranges[i - 1].second) return corrupt("tensor payload regions overlap");
  }
  return GFXB_OK;
}

// ---------------------------------------------------------------------------
// writer
// ---------------------------------------------------------------------------

StreamWriter::~StreamWriter() {
  if (fd_ >= 0) ::close(fd_);
  if (!finished_ && !temporary_.empty()) ::unlink(temporary_.c_str());
}

int StreamWriter::create(const char* path, const gfxb_artifact_identity& identity, const std::vector<Plan>& plans) {
  if (path == nullptr || path[0] == '\0') return fail(GFXB_INVALID_ARGUMENT, "artifact path is empty");
  if (plans.size() > std::numeric_limits<std::uint32_t>::max()) {
    return fail(GFXB_INVALID_ARGUMENT, "too many tensors for .gfxi v1");
  }
  if (!valid_identity_field(identity.target_arch) || !valid_identity_field(identity.model_id) ||
      !valid_identity_field(identity.weights_id) || !valid_identity_field(identity.recipe_id)) {
    return fail(GFXB_INVALID_ARGUMENT, "artifact identity is empty or too long");
  }
  std::unordered_map<std::string, int> seen;
  entries_.resize(plans.size());
  for (std::size_t i = 0; i < plans.size(); ++i) {
    const Plan& p = plans[i];
    if (!valid_name(p.name) || !seen.emplace(p.name, 0).second || p.dimensions.size() > 4 || p.data_bytes == 0 ||
        p.alignment < kFileAlignment || (p.alignment & (p.alignment - 1)) != 0) {
      const std::string message = "invalid tensor write request: " + p.name;
      return fail(GFXB_INVALID_ARGUMENT, message.c_str());
    }
    Tensor& e = entries_[i];
    e.name = p.name;
    e.dtype = p.dtype;
    e.quantization = p.quantization;
    e.rank = static_cast<std::uint16_t>(p.dimensions.size());
    e.alignment = p.alignment;
    for (std::size_t d = 0; d < p.dimensions.size(); ++d) e.dimensions[d] = p.dimensions[d];
    e.data_bytes = p.data_bytes;
    e.aux_bytes = p.aux_bytes;
    e.aux_offset = strings_.size();  // name offset until the payloads are placed
    strings_ += p.name;
  }
  const std::uint64_t directory_bytes = static_cast<std::uint64_t>(entries_.size()) * kEntryBytes;
  const std::uint64_t strings_offset = kHeaderBytes + directory_bytes;
  const std::uint64_t data_offset = align_up(strings_offset + strings_.size(), kFileAlignment);
  if (data_offset == 0) return fail(GFXB_INVALID_ARGUMENT, "artifact size overflow");
  std::uint64_t cursor = data_offset;
  std::vector<std::uint64_t> name_offsets(entries_.size());
  for (std::size_t i = 0; i < entries_.size(); ++i) {
    Tensor& e = entries_[i];
    name_offsets[i] = e.aux_offset;
    cursor = align_up(cursor, e.alignment);
    if (cursor == 0) return fail(GFXB_INVALID_ARGUMENT, "artifact payload offset overflow");
    e.data_offset = cursor;
    cursor += e.data_bytes;
    e.aux_offset = 0;
    if (e.aux_bytes != 0) {
      cursor = align_up(cursor, e.alignment);
      if (cursor == 0) return fail(GFXB_INVALID_ARGUMENT, "artifact auxiliary offset overflow");
      e.aux_offset = cursor;
      cursor += e.aux_bytes;
    }
  }
  header_.assign(kHeaderBytes + directory_bytes + strings_.size(), std::byte{0});
  std::byte* h = header_.data();
  std::memcpy(h, kMagic.data(), kMagic.size());
  put<std::uint32_t>(h, kHVersion, kVersion);
  put<std::uint32_t>(h, kHHeaderBytes, kHeaderBytes);
  put<std::uint32_t>(h, kHEndian, kEndianTag);
  put<std::uint64_t>(h, kHDirectory, kHeaderBytes);
  put<std::uint32_t>(h, kHTensorCount, static_cast<std::uint32_t>(entries_.size()));
  put<std::uint32_t>(h, kHEntryBytes, kEntryBytes);
  put<std::uint64_t>(h, kHStringsOffset, strings_offset);
  put<std::uint64_t>(h, kHStringsBytes, strings_.size());
  put<std::uint64_t>(h, kHDataOffset, data_offset);
  put<std::uint64_t>(h, kHDataBytes, cursor - data_offset);
  put<std::uint64_t>(h, kHFileBytes, cursor);
  std::memcpy(h + kHTargetArch, identity.target_arch, sizeof identity.target_arch);
  std::memcpy(h + kHModelId, identity.model_id, sizeof identity.model_id);
  std::memcpy(h + kHWeightsId, identity.weights_id, sizeof identity.weights_id);
  std::memcpy(h + kHRecipeId, identity.recipe_id, sizeof identity.recipe_id);
  for (std::size_t i = 0; i < entries_.size(); ++i) {
    std::byte* e = h + kHeaderBytes + i * kEntryBytes;
    const Tensor& t = entries_[i];
    put<std::uint64_t>(e, kENameOffset, name_offsets[i]);
    put<std::uint32_t>(e, kENameBytes, static_cast<std::uint32_t>(t.name.size()));
    put<std::uint16_t>(e, kEDtype, t.dtype);
    put<std::uint16_t>(e, kEQuant, t.quantization);
    put<std::uint16_t>(e, kERank, t.rank);
    put<std::uint32_t>(e, kEAlignment, t.alignment);
    for (int d = 0; d < 4; ++d) put<std::uint64_t>(e, kEDims + 8 * d, t.dimensions[d]);
    put<std::uint64_t>(e, kEDataOffset, t.data_offset);
    put<std::uint64_t>(e, kEDataBytes, t.data_bytes);
    put<std::uint64_t>(e, kEAuxOffset, t.aux_offset);
    put<std::uint64_t>(e, kEAuxBytes, t.aux_bytes);
  }
  std::memcpy(h + strings_offset, strings_.data(), strings_.size());

  path_ = path;
  temporary_ = path_ + ".tmp." + std::to_string(::getpid());
  fd_ = ::open(temporary_.c_str(), O_RDWR | O_CREAT | O_EXCL | O_CLOEXEC, 0644);
  if (fd_ < 0) {
    const std::string temporary = temporary_;
    temporary_.clear();  // not ours to unlink
    return io_error("cannot create", temporary);
  }
  if (::ftruncate(fd_, static_cast<off_t>(cursor)) != 0) return io_error("cannot size", temporary_);
  data_written_.assign(entries_.size(), 0);
  aux_written_.assign(entries_.size(), 0);
  data_crc_.assign(entries_.size(), 0);
  return GFXB_OK;
}

int StreamWriter::append(std::size_t index, bool aux, const void* bytes, std::uint64_t size) {
  if (fd_ < 0 || index >= entries_.size()) return fail(GFXB_INVALID_ARGUMENT, "artifact writer is not open");
  const Tensor& e = entries_[index];
  std::uint64_t& written = aux ? aux_written_[index] : data_written_[index];
  const std::uint64_t capacity = aux ? e.aux_bytes : e.data_bytes;
  if (size > capacity - written) return fail(GFXB_INVALID_ARGUMENT, "tensor payload exceeds its planned size");
  if (size == 0) return GFXB_OK;
  GFXB_TRY(write_at(fd_, bytes, size, (aux ? e.aux_offset : e.data_offset) + written));
  if (!aux) data_crc_[index] = crc64(data_crc_[index], bytes, static_cast<std::size_t>(size));
  written += size;
  return GFXB_OK;
}

int StreamWriter::finalize() {
  if (fd_ < 0) return fail(GFXB_INVALID_ARGUMENT, "artifact writer is not open");
  for (std::size_t i = 0; i < entries_.size(); ++i) {
    if (data_written_[i] != entries_[i].data_bytes || aux_written_[i] != entries_[i].aux_bytes) {
      const std::string message = "tensor payload is incomplete: " + entries_[i].name;
      return fail(GFXB_INVALID_ARGUMENT, message.c_str());
    }
    put<std::uint64_t>(header_.data() + kHeaderBytes + i * kEntryBytes, kEDataCrc, data_crc_[i]);
  }
  const std::size_t manifest = header_.size() - kHeaderBytes;
  put<std::uint64_t>(header_.data(), kHManifestCrc, crc64(0, header_.data() + kHeaderBytes, manifest));
  GFXB_TRY(write_at(fd_, header_.data(), header_.size(), 0));
  if (::fsync(fd_) != 0) return io_error("fsync failed for", temporary_);
  if (::close(fd_) != 0) {
    fd_ = -1;
    return io_error("close failed for", temporary_);
  }
  fd_ = -1;
  if (::rename(temporary_.c_str(), path_.c_str()) != 0) return io_error("cannot install artifact", path_);
  finished_ = true;
  return GFXB_OK;
}

}  // namespace gfxb::gfxi

// ===========================================================================
// C ABI
// ===========================================================================

struct gfxb_artifact {
  gfxb::gfxi::View view;
};

using gfxb::fail;

extern "C" int gfxb_crc64_ecma(std::uint64_t state, const void* bytes, std::size_t size, std::uint64_t* out) {
  if (out == nullptr || (bytes == nullptr && size != 0)) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  *out = gfxb::gfxi::crc64(state, bytes, size);
  return GFXB_OK;
}

extern "C" int gfxb_artifact_open(const char* path, int verify_checksums, gfxb_artifact** artifact) {
  if (path == nullptr || artifact == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  *artifact = nullptr;
  auto a = std::make_unique<gfxb_artifact>();
  GFXB_TRY(a->view.open(path, verify_checksums != 0));
  *artifact = a.release();
  return GFXB_OK;
}

extern "C" int gfxb_artifact_close(gfxb_artifact* artifact) {
  delete artifact;
  return GFXB_OK;
}

extern "C" int gfxb_artifact_identity_of(const gfxb_artifact* artifact, gfxb_artifact_identity* identity) {
  if (artifact == nullptr || identity == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  *identity = artifact->view.identity();
  return GFXB_OK;
}

extern "C" int gfxb_artifact_file_bytes(const gfxb_artifact* artifact, std::uint64_t* bytes) {
  if (artifact == nullptr || bytes == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  *bytes = artifact->view.file_bytes();
  return GFXB_OK;
}

extern "C" int gfxb_artifact_tensor_count(const gfxb_artifact* artifact, std::size_t* count) {
  if (artifact == nullptr || count == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  *count = artifact->view.tensors().size();
  return GFXB_OK;
}

extern "C" int gfxb_artifact_tensor_at(const gfxb_artifact* artifact, std::size_t index, gfxb_tensor_view* tensor) {
  if (artifact == nullptr || tensor == nullptr) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  if (index >= artifact->view.tensors().size()) return fail(GFXB_INVALID_ARGUMENT, "tensor index out of range");
  artifact->view.fill(artifact->view.tensors()[index], *tensor);
  return GFXB_OK;
}

extern "C" int gfxb_artifact_find(const gfxb_artifact* artifact, const char* name, gfxb_tensor_view* tensor,
                                  int* found) {
  if (artifact == nullptr || name == nullptr || tensor == nullptr || found == nullptr) {
    return fail(GFXB_INVALID_ARGUMENT, "null argument");
  }
  const gfxb::gfxi::Tensor* t = artifact->view.find(name);
  *found = t != nullptr;
  if (t != nullptr) artifact->view.fill(*t, *tensor);
  return GFXB_OK;
}

extern "C" int gfxb_artifact_write(const char* path, const gfxb_artifact_identity* identity,
                                   const gfxb_tensor_write* tensors, std::size_t count) {
  if (identity == nullptr || (tensors == nullptr && count != 0)) return fail(GFXB_INVALID_ARGUMENT, "null argument");
  std::vector<gfxb::gfxi::Plan> plans(count);
  for (std::size_t i = 0; i < count; ++i) {
    const gfxb_tensor_write& t = tensors[i];
    if (t.name == nullptr || t.rank > 4 || (t.data == nullptr && t.data_bytes != 0) ||
        (t.aux == nullptr && t.aux_bytes != 0)) {
      return fail(GFXB_INVALID_ARGUMENT, "invalid tensor write request");
    }
    plans[i].name = t.name;
    plans[i].dtype = t.dtype;
    plans[i].quantization = t.quantization;
    plans[i].dimensions.assign(t.dimensions, t.dimensions + t.rank);
    plans[i].data_bytes = t.data_bytes;
    plans[i].aux_bytes = t.aux_bytes;
    plans[i].alignment = t.alignment == 0 ? static_cast<std::uint32_t>(gfxb::gfxi::kFileAlignment) : t.alignment;
  }
  gfxb::gfxi::StreamWriter writer;
  GFXB_TRY(writer.create(path, *identity, plans));
  for (std::size_t i = 0; i < count; ++i) {
    GFXB_TRY(writer.append(i, false, tensors[i].data, tensors[i].data_bytes));
    GFXB_TRY(writer.append(i, true, tensors[i].aux, tensors[i].aux_bytes));
  }
  return writer.finalize();
}
