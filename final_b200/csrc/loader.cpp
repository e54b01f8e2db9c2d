// loader.cpp -- the reference's single-file model format, memory-mapped
// (include/b2loader.h).  Host C++ only.
//
// The reference's reader (src/model_loader.cpp) streams each tensor with
// ifstream::read into a fresh host Tensor and trusts the index; here the
// whole file is mapped once, every index entry is checked against the file
// size, and tensors are handed out as pointers into the mapping, so a model
// create that uploads from host memory reads the page cache directly.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/b2loader.h"

namespace {

struct Entry {
  std::string name;
  std::vector<int64_t> shape;
  uint64_t offset = 0;
  int64_t numel = 0;
  std::unique_ptr<float[]> aligned;  // copy when the offset is not 4-byte aligned
};

}  // namespace

struct b2_loader {
  int fd = -1;
  const uint8_t *base = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  std::vector<Entry> entries;
  std::unordered_map<std::string, size_t> index;
};

extern "C" b2_status b2_loader_close(b2_loader *l) {
  if (!l) return B2_OK;
  if (l->base) munmap(const_cast<uint8_t *>(l->base), l->size);
  if (l->fd >= 0) close(l->fd);
  delete l;
  return B2_OK;
}

extern "C" b2_status b2_loader_open(const char *path, b2_loader **out) {
  if (!path || !out) return B2_ERR_INVALID;
  *out = nullptr;
  b2_loader *l = new b2_loader();
  auto bad = [&]() {
    b2_loader_close(l);
    return B2_ERR_INVALID;
  };
  l->fd = open(path, O_RDONLY);
  if (l->fd < 0) return bad();
  struct stat st;
  if (fstat(l->fd, &st) != 0 || st.st_size < 12) return bad();
  l->size = (size_t)st.st_size;
  void *m = mmap(nullptr, l->size, PROT_READ, MAP_PRIVATE, l->fd, 0);
  if (m == MAP_FAILED) return bad();
  l->base = static_cast<const uint8_t *>(m);
  size_t pos = 0;
  auto rd = [&](void *dst, size_t n) {
    if (pos + n > l->size) return false;
    memcpy(dst, l->base + pos, n);
    pos += n;
    return true;
  };
  char magic[4];
  uint32_t n = 0;
  if (!rd(magic, 4) || memcmp(magic, "LFM2", 4) != 0) return bad();
  if (!rd(&l->version, 4) || !rd(&n, 4)) return bad();
  // every entry needs at least 4 + 1 + 4 + 8 bytes
  if ((uint64_t)n * 17 > l->size) return bad();
  l->entries.resize(n);
  for (uint32_t i = 0; i < n; ++i) {
    Entry &e = l->entries[i];
    uint32_t len = 0, ndim = 0;
    if (!rd(&len, 4) || len == 0 || len > 4096 || pos + len > l->size) return bad();
    e.name.assign(reinterpret_cast<const char *>(l->base + pos), len);
    pos += len;
    if (!rd(&ndim, 4) || ndim > 8) return bad();
    e.numel = 1;
    for (uint32_t d = 0; d < ndim; ++d) {
      uint32_t dim = 0;
      if (!rd(&dim, 4)) return bad();
      e.shape.push_back(dim);
      e.numel *= dim;
      if (e.numel > (int64_t)(l->size / 4)) return bad();
    }
    if (!rd(&e.offset, 8)) return bad();
    if (e.offset > l->size || (uint64_t)e.numel * 4 > l->size - e.offset) return bad();
    if (e.offset % 4 != 0 && e.numel > 0) {
      e.aligned.reset(new float[e.numel]);
      memcpy(e.aligned.get(), l->base + e.offset, (size_t)e.numel * 4);
    }
    l->index[e.name] = i;  // a repeated name keeps the last entry, as a map insert would
  }
  *out = l;
  return B2_OK;
}

extern "C" int64_t b2_loader_num_tensors(const b2_loader *l) {
  return l ? (int64_t)l->entries.size() : 0;
}

extern "C" const char *b2_loader_name(const b2_loader *l, int64_t i) {
  if (!l || i < 0 || i >= (int64_t)l->entries.size()) return nullptr;
  return l->entries[(size_t)i].name.c_str();
}

extern "C" b2_status b2_loader_tensor(const b2_loader *l, const char *name, const float **data,
                                      int64_t *numel, int64_t *shape, int *ndim) {
  if (!l || !name) return B2_ERR_INVALID;
  auto it = l->index.find(name);
  if (it == l->index.end()) return B2_ERR_INVALID;
  const Entry &e = l->entries[it->second];
  if (data)
    *data = e.aligned ? e.aligned.get() : reinterpret_cast<const float *>(l->base + e.offset);
  if (numel) *numel = e.numel;
  if (ndim) *ndim = (int)e.shape.size();
  if (shape)
    for (size_t d = 0; d < e.shape.size(); ++d) shape[d] = e.shape[d];
  return B2_OK;
}

extern "C" const float *b2_loader_weight(void *loader, const char *name, int64_t numel) {
  const float *p = nullptr;
  int64_t n = 0;
  if (b2_loader_tensor(static_cast<const b2_loader *>(loader), name, &p, &n, nullptr, nullptr) !=
      B2_OK)
    return nullptr;
  return n == numel ? p : nullptr;
}
