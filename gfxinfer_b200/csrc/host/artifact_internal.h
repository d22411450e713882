// `.gfxi` v1 container: the C++ side shared by the C ABI and
// the engine loader/exporter (runtime.cu); implemented in artifact.cu.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

#include "gfxb/artifact.h"

namespace gfxb::gfxi {

constexpr std::uint32_t kVersion = 1;
constexpr std::uint64_t kFileAlignment = 256;

std::uint64_t crc64(std::uint64_t state, const void* bytes, std::size_t size) noexcept;
bool valid_name(const std::string& name) noexcept;

struct Tensor {
  std::string name;
  std::uint16_t dtype = 0, quantization = 0, rank = 0, flags = 0;
  std::uint32_t alignment = 0;
  std::uint64_t dimensions[4] = {0, 0, 0, 0};
  std::uint64_t data_offset = 0, data_bytes = 0, aux_offset = 0, aux_bytes = 0, data_crc64 = 0;
};

// Read-only mapping of one artifact (ArtifactView, artifact.cpp:274-407).
class View {
 public:
  View() = default;
  ~View();
  View(const View&) = delete;
  View& operator=(const View&) = delete;

  int open(const char* path, bool verify_checksums);
  const gfxb_artifact_identity& identity() const { return identity_; }
  const std::vector<Tensor>& tensors() const { return tensors_; }
  const Tensor* find(const std::string& name) const;
  const std::byte* data(const Tensor& t) const { return mapping_ + t.data_offset; }
  const std::byte* aux(const Tensor& t) const { return t.aux_bytes != 0 ? mapping_ + t.aux_offset : nullptr; }
  std::uint64_t file_bytes() const { return bytes_; }
  void fill(const Tensor& t, gfxb_tensor_view& out) const;

 private:
  int fd_ = -1;
  const std::byte* mapping_ = nullptr;
  std::uint64_t bytes_ = 0;
  gfxb_artifact_identity identity_{};
  std::vector<Tensor> tensors_;
  std::unordered_map<std::string, std::size_t> index_;
};

struct Plan {
  std::string name;
  std::uint16_t dtype = 0, quantization = 0;
  std::vector<std::uint64_t> dimensions;
  std::uint64_t data_bytes = 0, aux_bytes = 0;
  std::uint32_t alignment = kFileAlignment;
};

// Writer whose payloads arrive in pieces (ArtifactStreamWriter,
// artifact.cpp:564-777): the layout is fixed by create(); append() writes
// each plane's bytes in order at their final offsets; finalize() writes the
// directory with the data checksums, fsyncs and renames the temporary file.
class StreamWriter {
 public:
  StreamWriter() = default;
  ~StreamWriter();
  StreamWriter(const StreamWriter&) = delete;
  StreamWriter& operator=(const StreamWriter&) = delete;

  int create(const char* path, const gfxb_artifact_identity& identity, const std::vector<Plan>& plans);
  int append(std::size_t index, bool aux, const void* bytes, std::uint64_t size);
  int finalize();

 private:
  int fd_ = -1;
  std::string path_, temporary_;
  std::vector<Tensor> entries_;
  std::vector<std::uint64_t> data_written_, aux_written_, data_crc_;
  std::string strings_;
  std::vector<std::byte> header_;
  bool finished_ = false;
};

}  // namespace gfxb::gfxi
