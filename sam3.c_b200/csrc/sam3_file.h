// sam3_file.h - reader of the .sam3 weight-file image (host only).
//
// The format is the reference's (src/core/weight.h:26-72, written by
// sam3_weight_write, weight.c:64-236): a 52-byte v4 header (48 bytes in v3),
// n_tensors 176-byte descriptors {name[128], dtype, n_dims, dims[4],
// data_offset, data_size, reserved}, then the data blob at the next 4096-byte
// boundary; every offset is relative to the blob.  The checks follow
// sam3_weight_open (weight.c:303-470).
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>

namespace s3 {

struct Sam3FileHeader {
  uint32_t magic, version, flags, n_tensors;
  int32_t image_size, encoder_dim, decoder_dim, n_encoder_layers, n_decoder_layers;
  uint32_t reserved[3];
  uint32_t text_backbone;  // v4 only
};
static_assert(sizeof(Sam3FileHeader) == 52, ".sam3 v4 header is 52 bytes");

struct Sam3FileDesc {
  char name[128];
  uint32_t dtype, n_dims;
  int32_t dims[4];
  uint64_t data_offset, data_size, reserved;
};
static_assert(sizeof(Sam3FileDesc) == 176, ".sam3 tensor descriptor is 176 bytes");

constexpr uint32_t kSam3Magic = 0x334D4153;  // "SAM3"

// A validated view of a file image; tensor data points into it.
struct Sam3File {
  const uint8_t* base = nullptr;
  size_t size = 0;
  const Sam3FileHeader* hdr = nullptr;
  const Sam3FileDesc* desc = nullptr;
  const uint8_t* data = nullptr;
  std::unordered_map<std::string, uint32_t> index;

  // 0, or SAM3CU_EINVAL (NULL image) / SAM3CU_EMODEL (malformed file).
  int open(const void* image, size_t bytes);
  const Sam3FileDesc* find(const char* name) const;
  const void* tensor_data(const Sam3FileDesc* d) const { return data + d->data_offset; }
  static int64_t numel(const Sam3FileDesc* d);
};

}  // namespace s3
