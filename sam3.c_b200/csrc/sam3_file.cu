// sam3_file.cu - the .sam3 weight-file reader and its C ABI
// (sam3cu_sam3_check / sam3cu_sam3_find).  Host code only.
#include <cstring>

#include "../../include/sam3cu.h"
#include "sam3_file.h"

namespace s3 {

int Sam3File::open(const void* image, size_t bytes) {
  if (!image) return SAM3CU_EINVAL;
  base = static_cast<const uint8_t*>(image);
  size = bytes;
  index.clear();
  if (bytes < 48) return SAM3CU_EMODEL;  // smaller than any header
  hdr = reinterpret_cast<const Sam3FileHeader*>(base);
  if (hdr->magic != kSam3Magic) return SAM3CU_EMODEL;
  size_t header_size;
  if (hdr->version == 3) header_size = 48;  // v3: no text_backbone word
  else if (hdr->version == 4) header_size = sizeof(Sam3FileHeader);
  else return SAM3CU_EMODEL;
  if (bytes < header_size) return SAM3CU_EMODEL;
  const uint64_t table_end = header_size + static_cast<uint64_t>(hdr->n_tensors) * sizeof(Sam3FileDesc);
  if (table_end > bytes) return SAM3CU_EMODEL;
  const uint64_t data_start = (table_end + 4095) & ~uint64_t(4095);
  if (data_start > bytes) return SAM3CU_EMODEL;
  desc = reinterpret_cast<const Sam3FileDesc*>(base + header_size);
  data = base + data_start;
  const uint64_t blob = bytes - data_start;
  index.reserve(hdr->n_tensors * 2);
  for (uint32_t i = 0; i < hdr->n_tensors; ++i) {
    const Sam3FileDesc& d = desc[i];
    if (d.data_offset > blob || d.data_size > blob - d.data_offset) return SAM3CU_EMODEL;
    // the first descriptor of a name wins: the reference inserts in file
    // order into a linear-probing table (weight.c:250-300), so its lookup
    // meets the earlier entry first
    index.emplace(std::string(d.name, strnlen(d.name, sizeof(d.name))), i);
  }
  return SAM3CU_OK;
}

const Sam3FileDesc* Sam3File::find(const char* name) const {
  if (!name) return nullptr;
  auto it = index.find(name);
  return it == index.end() ? nullptr : &desc[it->second];
}

int64_t Sam3File::numel(const Sam3FileDesc* d) {
  if (d->n_dims > 4) return -1;
  int64_t n = 1;
  for (uint32_t i = 0; i < d->n_dims; ++i) {
    if (d->dims[i] < 0) return -1;
    n *= d->dims[i];
  }
  return n;
}

}  // namespace s3

extern "C" {

int sam3cu_sam3_check(const void* image, size_t bytes, uint32_t* n_tensors, uint32_t* version) {
  s3::Sam3File f;
  const int rc = f.open(image, bytes);
  if (rc) return rc;
  if (n_tensors) *n_tensors = f.hdr->n_tensors;
  if (version) *version = f.hdr->version;
  return SAM3CU_OK;
}

int sam3cu_sam3_find(const void* image, size_t bytes, const char* name, int* dtype, int* n_dims, int* dims,
                     uint64_t* data_offset, uint64_t* nbytes) {
  s3::Sam3File f;
  int rc = f.open(image, bytes);
  if (rc) return rc;
  const s3::Sam3FileDesc* d = f.find(name);
  if (!d) return SAM3CU_ENOENT;
  if (dtype) *dtype = static_cast<int>(d->dtype);
  if (n_dims) *n_dims = static_cast<int>(d->n_dims);
  if (dims)
    for (int i = 0; i < 4; ++i) dims[i] = d->dims[i];
  // offset from the start of the image (not the blob), so the caller can
  // index its own mapping directly
  if (data_offset) *data_offset = static_cast<uint64_t>(f.data - f.base) + d->data_offset;
  if (nbytes) *nbytes = d->data_size;
  return SAM3CU_OK;
}

}  // extern "C"
