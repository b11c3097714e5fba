// ovw1.cpp -- the OVW1 weight-file reader of the C ABI (ovb_ovw1_*): map a
// file, validate its header and tensor index, look tensors up by name, check
// payload CRCs, and create device weights from int8 linear tensors straight
// out of the mapping.
//
// Format (the reference's docs/weight-format.en.md; reader
// cpp/src/core/weight_file.cpp:124-206): a 72-byte header (magic "OMNIVOIC",
// version 1, dtype_mode, n_tensors, header_bytes, index/names/data offsets,
// file_size, flags, n_params; 128 bytes reserved on disk), n 64-byte tensor
// descriptors at index_off (name offset/length, dtype 0 f32 / 1 i8 / 2 f16 /
// 3 i64, ndim, layout 0 row-major / 1 transposed [K, N], quant 0 / 1 per
// output channel, dims[4], aux_n, CRC32 in the low half of `hash`, payload
// offset and size, scale offset), names, payloads and fp32 scales.  The
// checks and their order follow the reference's reader so that a file it
// rejects is rejected here with the same reason.
//
// The reference prepares an int8 [N, K] tensor for its CPU kernels by
// repacking it into VNNI tiles on the host (s8_nk_pack, gemm.cpp:584-621,
// called by make_linear, mat.cpp:69-106), and its CUDA runner expands every
// int8 tensor to an fp32 device copy (LmRunner::weight, cuda_lm.cu:840-873).
// ovb_ovw1_weight instead copies the int8 payload as stored and packs it on
// the device (ovb_weight_create: either orientation, one K-major image).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdint>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "ovb200.h"
#include "ovb_internal.h"

namespace {

#pragma pack(push, 1)
struct OvwHeader {
  char magic[8];
  uint32_t version;
  uint32_t dtype_mode;
  uint32_t n_tensors;
  uint32_t header_bytes;
  uint64_t index_off;
  uint64_t names_off;
  uint64_t data_off;
  uint64_t file_size;
  uint64_t flags;
  uint64_t n_params;
};
struct OvwDesc {
  uint32_t name_off;
  uint32_t name_len;
  uint8_t dtype;
  uint8_t ndim;
  uint8_t layout;
  uint8_t quant;
  uint32_t dims[4];
  uint32_t aux_n;
  uint64_t hash;
  uint64_t data_off;
  uint64_t nbytes;
  uint64_t aux_off;
};
#pragma pack(pop)
static_assert(sizeof(OvwHeader) == 72, "OVW1 header fields");
static_assert(sizeof(OvwDesc) == 64, "OVW1 tensor descriptor");

constexpr uint32_t kOvwVersion = 1;

int64_t dtype_bytes(int dtype) {
  switch (dtype) {
    case 0: return 4;  // f32
    case 1: return 1;  // i8
    case 2: return 2;  // f16
    case 3: return 8;  // i64
    default: return 0;
  }
}

// CRC-32 (IEEE 802.3, reflected polynomial 0xEDB88320, initial value and
// final xor 0xFFFFFFFF), slicing by 8 bytes through eight 256-entry tables.
struct Crc32 {
  uint32_t t[8][256];
  Crc32() {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c >> 1) ^ (0xEDB88320u & (0u - (c & 1u)));
      t[0][i] = c;
    }
    for (uint32_t i = 0; i < 256; ++i)
      for (int s = 1; s < 8; ++s) t[s][i] = (t[s - 1][i] >> 8) ^ t[0][t[s - 1][i] & 0xFFu];
  }
  uint32_t operator()(const uint8_t* p, size_t n) const {
    uint32_t c = 0xFFFFFFFFu;
    while (n >= 8) {
      uint32_t lo, hi;
      std::memcpy(&lo, p, 4);
      std::memcpy(&hi, p + 4, 4);
      lo ^= c;
      c = t[7][lo & 0xFF] ^ t[6][(lo >> 8) & 0xFF] ^ t[5][(lo >> 16) & 0xFF] ^ t[4][lo >> 24] ^
          t[3][hi & 0xFF] ^ t[2][(hi >> 8) & 0xFF] ^ t[1][(hi >> 16) & 0xFF] ^ t[0][hi >> 24];
      p += 8;
      n -= 8;
    }
    while (n--) c = t[0][(c ^ *p++) & 0xFFu] ^ (c >> 8);
    return c ^ 0xFFFFFFFFu;
  }
};

const Crc32& crc_tables() {
  static const Crc32 c;
  return c;
}

}  // namespace

struct ovb_ovw1 {
  void* base = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  uint32_t dtype_mode = 0;
  uint64_t flags = 0;
  uint64_t n_params = 0;
  std::vector<ovb_ovw1_tensor> tensors;
  std::vector<std::string> names;  // owned copies (NUL-terminated)
  std::unordered_map<std::string, int64_t> index;
};

namespace {

int fail(const std::string& msg) {
  ovb::set_error("OVW1: " + msg);
  return OVB_ERR_INVALID_ARG;
}

void unmap(ovb_ovw1* f) {
  if (f->base) ::munmap(f->base, f->size);
  f->base = nullptr;
}

}  // namespace

extern "C" {

int ovb_ovw1_open(const char* path, ovb_ovw1** out) {
  if (!out) return fail("out is null");
  *out = nullptr;
  if (!path) return fail("path is null");
  const int fd = ::open(path, O_RDONLY);
  if (fd < 0) return fail(std::string("cannot open '") + path + "': " + std::strerror(errno));
  struct stat st {};
  if (::fstat(fd, &st) != 0) {
    ::close(fd);
    return fail(std::string("cannot stat '") + path + "'");
  }
  const size_t size = static_cast<size_t>(st.st_size);
  if (size < sizeof(OvwHeader)) {
    ::close(fd);
    return fail(std::string("'") + path + "' is smaller than a header");
  }
  void* base = ::mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (base == MAP_FAILED) return fail(std::string("mmap failed for '") + path + "'");
  auto* f = new ovb_ovw1();
  f->base = base;
  f->size = size;
  auto reject = [&](const std::string& msg) {
    unmap(f);
    delete f;
    return fail(msg);
  };

  OvwHeader h;
  std::memcpy(&h, base, sizeof h);
  if (std::memcmp(h.magic, "OMNIVOIC", 8) != 0) return reject("bad magic (not an OVW1 file)");
  if (h.version != kOvwVersion) return reject("unsupported version " + std::to_string(h.version));
  if (h.file_size != size)
    return reject("file size mismatch: header says " + std::to_string(h.file_size) +
                  ", actual " + std::to_string(size));
  const uint64_t index_end = h.index_off + static_cast<uint64_t>(h.n_tensors) * sizeof(OvwDesc);
  if (h.index_off < sizeof(OvwHeader) || index_end > size || index_end < h.index_off)
    return reject("index out of bounds");
  f->version = h.version;
  f->dtype_mode = h.dtype_mode;
  f->flags = h.flags;
  f->n_params = h.n_params;

  const char* cbase = static_cast<const char*>(base);
  f->tensors.reserve(h.n_tensors);
  f->names.reserve(h.n_tensors);
  for (uint32_t i = 0; i < h.n_tensors; ++i) {
    OvwDesc d;
    std::memcpy(&d, cbase + h.index_off + static_cast<uint64_t>(i) * sizeof(OvwDesc), sizeof d);
    const uint64_t name_begin = h.names_off + d.name_off;
    if (h.names_off > size || name_begin + d.name_len > size) return reject("tensor name out of bounds");
    if (d.data_off + d.nbytes > size || d.data_off + d.nbytes < d.data_off)
      return reject("tensor payload out of bounds");
    std::string name(cbase + name_begin, d.name_len);
    ovb_ovw1_tensor t = {};
    t.dtype = d.dtype;
    t.ndim = d.ndim;
    t.layout = d.layout;
    t.quant = d.quant;
    int64_t numel = 1;
    for (int k = 0; k < 4; ++k) {
      t.dims[k] = d.dims[k];
      if (k < d.ndim) numel *= static_cast<int64_t>(d.dims[k]);
    }
    t.data = cbase + d.data_off;
    t.nbytes = static_cast<int64_t>(d.nbytes);
    t.crc = static_cast<uint32_t>(d.hash & 0xFFFFFFFFu);
    if (d.quant == 1) {
      // Written so that no sum can wrap: a huge aux_off is out of bounds too.
      if (d.aux_off > size || static_cast<uint64_t>(d.aux_n) * 4 > size - d.aux_off)
        return reject("scales out of bounds");
      t.scales = reinterpret_cast<const float*>(cbase + d.aux_off);
      t.n_scales = d.aux_n;
    }
    const int64_t expect = numel * dtype_bytes(d.dtype);
    if (expect != t.nbytes) {
      std::string shape = "[";
      for (int k = 0; k < d.ndim && k < 4; ++k)
        shape += (k ? ", " : "") + std::to_string(static_cast<int32_t>(d.dims[k]));
      return reject("size mismatch for '" + name + "': shape " + shape + "] needs " +
                    std::to_string(expect) + " bytes, descriptor says " + std::to_string(t.nbytes));
    }
    f->index.emplace(name, static_cast<int64_t>(f->tensors.size()));
    f->names.push_back(std::move(name));
    f->tensors.push_back(t);
  }
  for (size_t i = 0; i < f->tensors.size(); ++i) {
    f->tensors[i].name = f->names[i].c_str();
    f->tensors[i].name_len = static_cast<int32_t>(f->names[i].size());
  }
  *out = f;
  return OVB_OK;
}

int ovb_ovw1_close(ovb_ovw1* f) {
  if (!f) return OVB_OK;
  unmap(f);
  delete f;
  return OVB_OK;
}

int64_t ovb_ovw1_count(const ovb_ovw1* f) {
  return f ? static_cast<int64_t>(f->tensors.size()) : 0;
}

int ovb_ovw1_header(const ovb_ovw1* f, uint32_t* dtype_mode, uint64_t* flags, uint64_t* n_params) {
  if (!f) return fail("file is null");
  if (dtype_mode) *dtype_mode = f->dtype_mode;
  if (flags) *flags = f->flags;
  if (n_params) *n_params = f->n_params;
  return OVB_OK;
}

int ovb_ovw1_tensor_at(const ovb_ovw1* f, int64_t i, ovb_ovw1_tensor* out) {
  if (!f || !out) return fail("file/out is null");
  if (i < 0 || i >= static_cast<int64_t>(f->tensors.size())) return fail("tensor index out of range");
  *out = f->tensors[static_cast<size_t>(i)];
  return OVB_OK;
}

int ovb_ovw1_find(const ovb_ovw1* f, const char* name, ovb_ovw1_tensor* out) {
  if (!f || !name || !out) return fail("file/name/out is null");
  auto it = f->index.find(name);
  if (it == f->index.end()) return fail(std::string("tensor not found: '") + name + "'");
  *out = f->tensors[static_cast<size_t>(it->second)];
  return OVB_OK;
}

int ovb_ovw1_crc(const ovb_ovw1* f, const char* name, uint32_t* computed) {
  if (!computed) return fail("computed is null");
  ovb_ovw1_tensor t;
  const int rc = ovb_ovw1_find(f, name, &t);
  if (rc != OVB_OK) return rc;
  *computed = crc_tables()(static_cast<const uint8_t*>(t.data), static_cast<size_t>(t.nbytes));
  return OVB_OK;
}

namespace {

// The ovb_weight_src of an int8 linear tensor (make_linear's checks,
// mat.cpp:69-106), or a status.
int linear_src(const ovb_ovw1* f, const char* name, ovb_weight_src* src) {
  ovb_ovw1_tensor t;
  const int rc = ovb_ovw1_find(f, name, &t);
  if (rc != OVB_OK) return rc;
  if (t.ndim != 2) return fail(std::string(name) + ": expected a 2-D weight");
  if (t.dtype != 1 || t.quant != 1 || !t.scales)
    return fail(std::string(name) + ": not an int8 weight with per-output-channel scales");
  // layout 1: [K, N] with one scale per column; layout 0: [N, K], one per row
  const bool kn = t.layout == 1;
  src->W = static_cast<const int8_t*>(t.data);
  src->layout = kn ? OVB_LAYOUT_KN : OVB_LAYOUT_NK;
  src->N = kn ? t.dims[1] : t.dims[0];
  src->K = kn ? t.dims[0] : t.dims[1];
  src->scale = t.scales;
  if (t.n_scales != src->N) return fail(std::string(name) + ": scale count != N");
  return OVB_OK;
}

}  // namespace

int ovb_ovw1_weights(const ovb_ovw1* f, const char* const* names, int n, int flags, void* stream,
                     ovb_weight** out) {
  if (!out) return fail("out is null");
  if (n < 0 || (n > 0 && !names)) return fail("names/n");
  if ((flags & ~OVB_WEIGHT_F16) != 0) return fail("flags: only OVB_WEIGHT_F16 applies");
  std::vector<ovb_weight_src> srcs(static_cast<size_t>(n));
  for (int i = 0; i < n; ++i) {
    out[i] = nullptr;
    const int rc = linear_src(f, names[i], &srcs[static_cast<size_t>(i)]);
    if (rc != OVB_OK) return rc;
  }
  if (n == 0) return OVB_OK;
  // Copies straight from the mapping.  (Page-locking the mapping first with
  // cudaHostRegister made a 440 MB load 4-8x slower than these pageable
  // copies, measured on the B200 hosts.)
  return ovb_weight_create_batch(srcs.data(), n, flags & OVB_WEIGHT_F16, stream, out);
}

int ovb_ovw1_weight(const ovb_ovw1* f, const char* name, int flags, void* stream,
                    ovb_weight** out) {
  if (!out) return fail("out is null");
  *out = nullptr;
  ovb_weight_src src;
  const int rc = linear_src(f, name, &src);
  if (rc != OVB_OK) return rc;
  if ((flags & ~OVB_WEIGHT_F16) != 0) return fail("flags: only OVB_WEIGHT_F16 applies");
  return ovb_weight_create(src.W, src.layout, src.N, src.K, src.scale, flags & OVB_WEIGHT_F16,
                           stream, out);
}

}  // extern "C"
