// GGUF tensor-view loader: mmap + parse of a .gguf file and staged copies of raw tensor bytes into
// device memory (include/gguf_file.h).  Host code only; the ops of gguf_ops.h consume the copied
// bytes as they lie in the file.
//
// Parse rules follow gguf-py 0.19.0's GGUFReader (gguf/gguf_reader.py:111-186, :221-316, :318-360):
// versions 2 and 3, u64 counts, general.alignment must be a UINT32 non-zero power of two (default
// 32), the data section starts at the header end rounded up to it, tensor sizes are
// n_elements / block * type_size, duplicate tensor names and duplicate keys are errors.  Stricter
// than the reader where a device copy needs it: every section and every tensor's bytes must lie
// inside the file, rows must hold whole blocks, and at most 4 dims (ggml's GGML_MAX_DIMS).
// Big-endian files (which the reader byte-swaps) are rejected.

#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "gguf_file.h"

namespace gguf_b200 {
int set_error(int code, const std::string& msg);  // gguf_ops.cu: fills gguf_last_error()
void clear_error();
}  // namespace gguf_b200

using gguf_b200::set_error;

struct GgufFile {
  int fd = -1;
  const uint8_t* base = nullptr;
  size_t size = 0;
  int32_t version = 0;
  int64_t alignment = 32;
  int64_t data_offset = 0;
  std::vector<std::string> keys, names;
  std::vector<GgufKv> kvs;
  std::vector<GgufTensorInfo> tensors;
  std::unordered_map<std::string, int64_t> kv_index, tensor_index;

  // upload staging (lazily allocated on the first upload)
  std::mutex upload_mu;
  static constexpr int kStages = 4;
  static constexpr size_t kChunk = size_t(32) << 20;
  void* stage[kStages] = {};
  cudaEvent_t done[kStages] = {};
  bool pending[kStages] = {};
  int stage_device = -1;
};

namespace {

// ggml block size and bytes per block by type id (gguf/constants.py GGML_QUANT_SIZES).
struct TypeSize {
  int32_t id;
  int64_t block, bytes;
};
constexpr TypeSize kTypes[] = {
    {0, 1, 4},      {1, 1, 2},      {2, 32, 18},    {3, 32, 20},    {6, 32, 22},    {7, 32, 24},
    {8, 32, 34},    {9, 32, 40},    {10, 256, 84},  {11, 256, 110}, {12, 256, 144}, {13, 256, 176},
    {14, 256, 210}, {15, 256, 292}, {16, 256, 66},  {17, 256, 74},  {18, 256, 98},  {19, 256, 50},
    {20, 32, 18},   {21, 256, 110}, {22, 256, 82},  {23, 256, 136}, {24, 1, 1},     {25, 1, 2},
    {26, 1, 4},     {27, 1, 8},     {28, 1, 8},     {29, 256, 56},  {30, 1, 2},     {34, 256, 54},
    {35, 256, 66},  {39, 32, 17},   {40, 64, 36},   {41, 128, 18}};

const TypeSize* find_type(int32_t id) {
  for (const auto& t : kTypes)
    if (t.id == id) return &t;
  return nullptr;
}

// Bytes of a scalar metadata value type; 0 for STRING / ARRAY / unknown.
int64_t scalar_bytes(uint32_t t) {
  switch (t) {
    case GGUF_VAL_UINT8: case GGUF_VAL_INT8: case GGUF_VAL_BOOL: return 1;
    case GGUF_VAL_UINT16: case GGUF_VAL_INT16: return 2;
    case GGUF_VAL_UINT32: case GGUF_VAL_INT32: case GGUF_VAL_FLOAT32: return 4;
    case GGUF_VAL_UINT64: case GGUF_VAL_INT64: case GGUF_VAL_FLOAT64: return 8;
    default: return 0;
  }
}

// Bounds-checked little-endian reader over the mapping.
struct Cursor {
  const uint8_t* p;
  size_t size, pos = 0;
  std::string err;

  bool need(size_t n, const char* what) {
    if (!err.empty()) return false;
    if (n > size - pos) {
      err = std::string("GGUF: truncated file while reading ") + what + " at byte " + std::to_string(pos);
      return false;
    }
    return true;
  }
  template <typename T>
  bool get(T& v, const char* what) {
    if (!need(sizeof(T), what)) return false;
    std::memcpy(&v, p + pos, sizeof(T));
    pos += sizeof(T);
    return true;
  }
  bool str(std::string* out, const char* what) {
    uint64_t n;
    if (!get(n, what) || !need(n, what)) return false;
    if (out) out->assign(reinterpret_cast<const char*>(p + pos), n);
    pos += n;
    return true;
  }
  // Skips one value of type t (nested arrays included), depth-limited.
  bool skip_value(uint32_t t, int depth) {
    if (depth > 8) {
      err = "GGUF: metadata arrays nested too deeply";
      return false;
    }
    if (const int64_t b = scalar_bytes(t)) return need(b, "metadata value") && (pos += b, true);
    if (t == GGUF_VAL_STRING) return str(nullptr, "metadata string");
    if (t == GGUF_VAL_ARRAY) {
      uint32_t et;
      uint64_t n;
      if (!get(et, "array type") || !get(n, "array length")) return false;
      if (const int64_t b = scalar_bytes(et)) {
        if (n > (size - pos) / b) {
          err = "GGUF: truncated file while reading a metadata array at byte " + std::to_string(pos);
          return false;
        }
        pos += n * b;
        return true;
      }
      for (uint64_t i = 0; i < n; ++i)
        if (!skip_value(et, depth + 1)) return false;
      return true;
    }
    err = "GGUF: unknown metadata value type " + std::to_string(t);
    return false;
  }
};

int parse(GgufFile* f) {
  Cursor c{f->base, f->size};
  uint32_t magic, version;
  if (!c.get(magic, "magic") || magic != 0x46554747u)  // "GGUF"
    return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: bad magic (not a GGUF file)");
  if (!c.get(version, "version")) return set_error(GGUF_ERR_INVALID_ARGUMENT, c.err);
  if ((version & 0xFFFFu) == 0)
    return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: big-endian files are not supported");
  if (version != 2 && version != 3)
    return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: unsupported version " + std::to_string(version));
  f->version = static_cast<int32_t>(version);
  uint64_t n_tensors, n_kv;
  if (!c.get(n_tensors, "tensor count") || !c.get(n_kv, "kv count"))
    return set_error(GGUF_ERR_INVALID_ARGUMENT, c.err);
  // every kv takes >= 12 bytes and every tensor info >= 24: counts beyond that are truncation
  if (n_kv > f->size / 12 || n_tensors > f->size / 24)
    return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: truncated file (counts exceed the file size)");

  f->keys.reserve(n_kv);
  f->kvs.reserve(n_kv);
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key;
    uint32_t t;
    if (!c.str(&key, "metadata key") || !c.get(t, "metadata type")) return set_error(GGUF_ERR_INVALID_ARGUMENT, c.err);
    GgufKv kv{};
    kv.type = static_cast<int32_t>(t);
    kv.elem_type = -1;
    const size_t start = c.pos;
    if (t == GGUF_VAL_STRING) {
      uint64_t n;
      if (!c.get(n, "metadata string")) return set_error(GGUF_ERR_INVALID_ARGUMENT, c.err);
      kv.count = static_cast<int64_t>(n);
      c.pos = start;
    } else if (t == GGUF_VAL_ARRAY) {
      uint32_t et;
      uint64_t n;
      if (!c.get(et, "array type") || !c.get(n, "array length")) return set_error(GGUF_ERR_INVALID_ARGUMENT, c.err);
      kv.elem_type = static_cast<int32_t>(et);
      kv.count = static_cast<int64_t>(n);
      c.pos = start;
    } else {
      kv.count = 1;
    }
    if (!c.skip_value(t, 0)) return set_error(GGUF_ERR_INVALID_ARGUMENT, c.err);
    const size_t hdr = t == GGUF_VAL_STRING ? 8 : t == GGUF_VAL_ARRAY ? 12 : 0;
    kv.data = f->base + start + hdr;
    kv.nbytes = static_cast<int64_t>(c.pos - start - hdr);
    if (!f->kv_index.emplace(key, static_cast<int64_t>(f->kvs.size())).second)
      return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: duplicate metadata key " + key);
    f->keys.push_back(std::move(key));
    f->kvs.push_back(kv);
  }
  for (size_t i = 0; i < f->kvs.size(); ++i) f->kvs[i].key = f->keys[i].c_str();

  f->names.reserve(n_tensors);
  f->tensors.reserve(n_tensors);
  std::vector<uint64_t> rel(n_tensors);
  for (uint64_t i = 0; i < n_tensors; ++i) {
    std::string name;
    uint32_t nd, type;
    GgufTensorInfo ti{};
    if (!c.str(&name, "tensor name") || !c.get(nd, "tensor dims")) return set_error(GGUF_ERR_INVALID_ARGUMENT, c.err);
    if (nd < 1 || nd > 4)
      return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: tensor " + name + " has " + std::to_string(nd) +
                                                      " dims (1..4 supported)");
    ti.n_dims = static_cast<int32_t>(nd);
    int64_t elems = 1;
    for (int d = 0; d < 4; ++d) ti.dims[d] = 1;
    for (uint32_t d = 0; d < nd; ++d) {
      uint64_t v;
      if (!c.get(v, "tensor dim")) return set_error(GGUF_ERR_INVALID_ARGUMENT, c.err);
      if (v > (uint64_t(1) << 40) || (v && static_cast<uint64_t>(elems) > (uint64_t(1) << 62) / v))
        return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: tensor " + name + " is too large");
      ti.dims[d] = static_cast<int64_t>(v);
      elems *= static_cast<int64_t>(v);
    }
    uint64_t off;
    if (!c.get(type, "tensor type") || !c.get(off, "tensor offset")) return set_error(GGUF_ERR_INVALID_ARGUMENT, c.err);
    const TypeSize* ts = find_type(static_cast<int32_t>(type));
    if (!ts)
      return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: tensor " + name + " has unknown type " + std::to_string(type));
    if (ti.dims[0] % ts->block != 0)
      return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: tensor " + name + " rows are not whole blocks");
    ti.type = static_cast<int32_t>(type);
    ti.block_elems = ts->block;
    ti.block_bytes = ts->bytes;
    // the byte size must fit int64 (a malformed file can claim up to 2^62 elements of a type with
    // several bytes per element); anything larger than the file is rejected later anyway
    int64_t nbytes = 0;
    if (__builtin_mul_overflow(elems / ts->block, static_cast<int64_t>(ts->bytes), &nbytes))
      return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: tensor " + name + " is too large");
    ti.row_bytes = ti.dims[0] / ts->block * ts->bytes;
    ti.nbytes = nbytes;
    rel[i] = off;
    if (!f->tensor_index.emplace(name, static_cast<int64_t>(f->tensors.size())).second)
      return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: duplicate tensor name " + name);
    f->names.push_back(std::move(name));
    f->tensors.push_back(ti);
  }

  auto it = f->kv_index.find("general.alignment");
  if (it != f->kv_index.end()) {
    const GgufKv& kv = f->kvs[it->second];
    if (kv.type != GGUF_VAL_UINT32) return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: bad type for general.alignment");
    uint32_t a;
    std::memcpy(&a, kv.data, 4);
    if (a == 0 || (a & (a - 1)) != 0)
      return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: invalid alignment (must be a non-zero power of two)");
    f->alignment = a;
  }
  const uint64_t data = (c.pos + f->alignment - 1) / f->alignment * f->alignment;
  f->data_offset = static_cast<int64_t>(data);
  for (size_t i = 0; i < f->tensors.size(); ++i) {
    GgufTensorInfo& ti = f->tensors[i];
    ti.name = f->names[i].c_str();
    if (rel[i] > f->size || data + rel[i] > f->size || static_cast<uint64_t>(ti.nbytes) > f->size - data - rel[i])
      return set_error(GGUF_ERR_INVALID_ARGUMENT, std::string("GGUF: data of tensor ") + ti.name +
                                                      " lies beyond the end of the file");
    ti.offset = static_cast<int64_t>(data + rel[i]);
  }
  return GGUF_OK;
}

void release_staging(GgufFile* f) {
  for (int s = 0; s < GgufFile::kStages; ++s) {
    if (f->done[s]) {
      if (f->pending[s]) cudaEventSynchronize(f->done[s]);
      cudaEventDestroy(f->done[s]);
      f->done[s] = nullptr;
    }
    if (f->stage[s]) {
      cudaFreeHost(f->stage[s]);
      f->stage[s] = nullptr;
    }
    f->pending[s] = false;
  }
  f->stage_device = -1;
}

int cuda_error(const char* what, cudaError_t e) {
  return set_error(GGUF_ERR_CUDA, std::string("GGUF upload: ") + what + ": " + cudaGetErrorString(e));
}

// Copies n bytes host -> host with up to `threads` threads (page faults of the mapping are taken in
// parallel; one thread per >= 4 MiB).
void parallel_copy(void* dst, const uint8_t* src, size_t n, unsigned threads) {
  const size_t per = size_t(4) << 20;
  const unsigned k = static_cast<unsigned>(std::max<size_t>(1, std::min<size_t>(threads, (n + per - 1) / per)));
  if (k == 1) {
    std::memcpy(dst, src, n);
    return;
  }
  std::vector<std::thread> pool;
  pool.reserve(k - 1);
  const size_t part = (n + k - 1) / k;
  for (unsigned i = 1; i < k; ++i) {
    const size_t lo = std::min(n, i * part), hi = std::min(n, lo + part);
    pool.emplace_back([=] { std::memcpy(static_cast<uint8_t*>(dst) + lo, src + lo, hi - lo); });
  }
  std::memcpy(dst, src, std::min(n, part));
  for (auto& t : pool) t.join();
}

}  // namespace

extern "C" {

int gguf_type_size(int32_t type, int64_t* block_elems, int64_t* block_bytes) {
  gguf_b200::clear_error();
  const TypeSize* t = find_type(type);
  if (!t) return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: unknown type " + std::to_string(type));
  if (block_elems) *block_elems = t->block;
  if (block_bytes) *block_bytes = t->bytes;
  return GGUF_OK;
}

int gguf_file_open(const char* path, GgufFile** out) {
  gguf_b200::clear_error();
  if (!out || !path) return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: null argument");
  *out = nullptr;
  const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return set_error(GGUF_ERR_IO, std::string("GGUF: cannot open ") + path + ": " + std::strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size <= 0) {
    ::close(fd);
    return set_error(GGUF_ERR_INVALID_ARGUMENT, std::string("GGUF: empty or unreadable file ") + path);
  }
  void* m = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_SHARED, fd, 0);
  if (m == MAP_FAILED) {
    ::close(fd);
    return set_error(GGUF_ERR_IO, std::string("GGUF: cannot map ") + path + ": " + std::strerror(errno));
  }
  madvise(m, static_cast<size_t>(st.st_size), MADV_SEQUENTIAL);
  auto* f = new GgufFile;
  f->fd = fd;
  f->base = static_cast<const uint8_t*>(m);
  f->size = static_cast<size_t>(st.st_size);
  const int rc = parse(f);
  if (rc != GGUF_OK) {
    gguf_file_close(f);
    return rc;
  }
  *out = f;
  return GGUF_OK;
}

void gguf_file_close(GgufFile* f) {
  if (!f) return;
  release_staging(f);
  if (f->base) munmap(const_cast<uint8_t*>(f->base), f->size);
  if (f->fd >= 0) ::close(f->fd);
  delete f;
}

int gguf_file_header(const GgufFile* f, int32_t* version, int64_t* alignment, int64_t* data_offset,
                     int64_t* file_size) {
  if (!f) return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: null handle");
  if (version) *version = f->version;
  if (alignment) *alignment = f->alignment;
  if (data_offset) *data_offset = f->data_offset;
  if (file_size) *file_size = static_cast<int64_t>(f->size);
  return GGUF_OK;
}

const void* gguf_file_data(const GgufFile* f) { return f ? f->base : nullptr; }

int64_t gguf_file_tensor_count(const GgufFile* f) { return f ? static_cast<int64_t>(f->tensors.size()) : 0; }

int gguf_file_tensor_info(const GgufFile* f, int64_t i, GgufTensorInfo* out) {
  if (!f || !out || i < 0 || i >= static_cast<int64_t>(f->tensors.size()))
    return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: tensor index out of range");
  *out = f->tensors[static_cast<size_t>(i)];
  return GGUF_OK;
}

int64_t gguf_file_find_tensor(const GgufFile* f, const char* name) {
  if (!f || !name) return -1;
  auto it = f->tensor_index.find(name);
  return it == f->tensor_index.end() ? -1 : it->second;
}

int64_t gguf_file_kv_count(const GgufFile* f) { return f ? static_cast<int64_t>(f->kvs.size()) : 0; }

int gguf_file_kv(const GgufFile* f, int64_t i, GgufKv* out) {
  if (!f || !out || i < 0 || i >= static_cast<int64_t>(f->kvs.size()))
    return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF: metadata index out of range");
  *out = f->kvs[static_cast<size_t>(i)];
  return GGUF_OK;
}

int64_t gguf_file_find_kv(const GgufFile* f, const char* key) {
  if (!f || !key) return -1;
  auto it = f->kv_index.find(key);
  return it == f->kv_index.end() ? -1 : it->second;
}

int gguf_file_upload(GgufFile* f, const GgufUploadItem* items, int64_t n, void* stream) {
  gguf_b200::clear_error();
  if (!f) return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF upload: null handle");
  if (n < 0 || (n > 0 && !items)) return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF upload: bad item list");
  for (int64_t i = 0; i < n; ++i) {
    const GgufUploadItem& it = items[i];
    if (it.tensor < 0 || it.tensor >= static_cast<int64_t>(f->tensors.size()))
      return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF upload: tensor index out of range");
    const int64_t tb = f->tensors[static_cast<size_t>(it.tensor)].nbytes;
    const int64_t len = it.nbytes < 0 ? tb - it.byte_offset : it.nbytes;
    if (it.byte_offset < 0 || it.byte_offset > tb || len > tb - it.byte_offset)
      return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF upload: byte range outside the tensor");
    if (len > 0 && !it.dst) return set_error(GGUF_ERR_INVALID_ARGUMENT, "GGUF upload: null destination");
  }
  std::lock_guard<std::mutex> lock(f->upload_mu);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error("cudaGetDevice", e);
  if (f->stage_device != dev) {  // (re)allocate the staging ring for this device
    release_staging(f);
    for (int s = 0; s < GgufFile::kStages; ++s) {
      if ((e = cudaHostAlloc(&f->stage[s], GgufFile::kChunk, cudaHostAllocDefault)) != cudaSuccess ||
          (e = cudaEventCreateWithFlags(&f->done[s], cudaEventDisableTiming)) != cudaSuccess) {
        release_staging(f);
        return cuda_error("staging allocation", e);
      }
    }
    f->stage_device = dev;
  }
  const unsigned threads = std::max(1u, std::min(16u, std::thread::hardware_concurrency() / 2));
  auto* s = static_cast<cudaStream_t>(stream);
  int slot = 0;
  int rc = GGUF_OK;
  for (int64_t i = 0; i < n && rc == GGUF_OK; ++i) {
    const GgufUploadItem& it = items[i];
    const GgufTensorInfo& ti = f->tensors[static_cast<size_t>(it.tensor)];
    int64_t len = it.nbytes < 0 ? ti.nbytes - it.byte_offset : it.nbytes;
    const uint8_t* src = f->base + ti.offset + it.byte_offset;
    auto* dst = static_cast<uint8_t*>(it.dst);
    while (len > 0) {
      const size_t chunk = static_cast<size_t>(std::min<int64_t>(len, static_cast<int64_t>(GgufFile::kChunk)));
      if (f->pending[slot]) {
        if ((e = cudaEventSynchronize(f->done[slot])) != cudaSuccess) {
          rc = cuda_error("staging wait", e);
          break;
        }
        f->pending[slot] = false;
      }
      parallel_copy(f->stage[slot], src, chunk, threads);
      if ((e = cudaMemcpyAsync(dst, f->stage[slot], chunk, cudaMemcpyHostToDevice, s)) != cudaSuccess ||
          (e = cudaEventRecord(f->done[slot], s)) != cudaSuccess) {
        rc = cuda_error("cudaMemcpyAsync", e);
        break;
      }
      f->pending[slot] = true;
      slot = (slot + 1) % GgufFile::kStages;
      src += chunk;
      dst += chunk;
      len -= static_cast<int64_t>(chunk);
    }
  }
  for (int k = 0; k < GgufFile::kStages; ++k) {  // every copy done: staging free, bytes on the device
    if (!f->pending[k]) continue;
    e = cudaEventSynchronize(f->done[k]);
    f->pending[k] = false;
    if (e != cudaSuccess && rc == GGUF_OK) rc = cuda_error("staging wait", e);
  }
  return rc;
}

}  // extern "C"
