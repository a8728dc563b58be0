// kq_gguf.cu -- GGUF file reader: header, metadata, tensor directory, tensor
// bytes, and upload of K-quant tensors as device-resident kq_weights.
//
// pesti reaches GGUF files through the external pesti-gguf crate
// (extract_tensor_bytes_from_path, called at pesti-runner/src/
// gguf_weight_loader.rs:79-81, the GgufDtype / stored_size helpers at :20-21)
// and keeps the raw tensor bytes (:73-89) before materialising f32 copies.
// Here the raw bytes of a Q4_K / Q6_K tensor go straight to kq_weight_upload:
// one host read, one copy to HBM, no f32 copy anywhere.
//
// Layout read (GGUF versions 2 and 3, little-endian):
//   u32 magic "GGUF", u32 version, u64 tensor count, u64 metadata count;
//   metadata: string key, u32 value type, value (scalars, strings = u64 length
//   + bytes, arrays = u32 element type + u64 count + elements);
//   tensor directory: string name, u32 n_dims, u64 ne[n_dims] (ne[0] the
//   innermost), u32 ggml type, u64 offset from the data section;
//   data section at the next multiple of general.alignment (default 32).
// Every length and offset is checked against the file size before it is
// used; a malformed file is an error (KQ_ERR_FORMAT), never a crash.  Host
// code only (no kernels).
#include "pesti_kq.h"

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <set>
#include <string>
#include <vector>

namespace {

enum : uint32_t {
  GV_U8 = 0, GV_I8, GV_U16, GV_I16, GV_U32, GV_I32, GV_F32, GV_BOOL, GV_STRING, GV_ARRAY, GV_U64, GV_I64, GV_F64
};

// bytes of one scalar metadata value, 0 for strings / arrays / unknown types
uint64_t scalar_bytes(uint32_t t) {
  switch (t) {
    case GV_U8: case GV_I8: case GV_BOOL: return 1;
    case GV_U16: case GV_I16: return 2;
    case GV_U32: case GV_I32: case GV_F32: return 4;
    case GV_U64: case GV_I64: case GV_F64: return 8;
    default: return 0;
  }
}

// (elements per block, bytes per block) of the ggml tensor types whose size
// the reader computes; 0 for types it lists but does not size
void ggml_block(uint32_t type, uint64_t& elems, uint64_t& bytes) {
  elems = 0;
  bytes = 0;
  switch (type) {
    case 0: elems = 1; bytes = 4; break;      // F32
    case 1: elems = 1; bytes = 2; break;      // F16
    case 30: elems = 1; bytes = 2; break;     // BF16
    case 2: elems = 32; bytes = 18; break;    // Q4_0
    case 3: elems = 32; bytes = 20; break;    // Q4_1
    case 6: elems = 32; bytes = 22; break;    // Q5_0
    case 7: elems = 32; bytes = 24; break;    // Q5_1
    case 8: elems = 32; bytes = 34; break;    // Q8_0
    case 10: elems = 256; bytes = 84; break;  // Q2_K
    case 11: elems = 256; bytes = 110; break; // Q3_K
    case 12: elems = 256; bytes = 144; break; // Q4_K
    case 13: elems = 256; bytes = 176; break; // Q5_K
    case 14: elems = 256; bytes = 210; break; // Q6_K
    case 15: elems = 256; bytes = 292; break; // Q8_K
    default: break;
  }
}

struct Meta {
  std::string key;
  uint32_t type = 0, elem_type = 0;
  uint64_t count = 1;              // 1 for a scalar or a string, the element count for an array
  std::vector<uint8_t> data;       // scalar / packed scalar array bytes (little-endian)
  std::vector<std::string> strs;   // a string, or the elements of a string array
};

struct Tensor {
  std::string name;
  uint32_t type = 0, n_dims = 0;
  int64_t ne[4] = {1, 1, 1, 1};
  uint64_t offset = 0, nbytes = 0;  // absolute file offset; 0 bytes when the type is not sized
};

class Reader {
 public:
  Reader(FILE* f, uint64_t size) : f_(f), size_(size) {}
  uint64_t pos() const { return pos_; }
  bool bytes(void* dst, uint64_t n) {
    if (n > size_ - pos_ || (n && fread(dst, 1, (size_t)n, f_) != (size_t)n)) return false;
    pos_ += n;
    return true;
  }
  bool skip(uint64_t n) {
    if (n > size_ - pos_ || fseeko(f_, (off_t)n, SEEK_CUR) != 0) return false;
    pos_ += n;
    return true;
  }
  template <class T>
  bool get(T& v) {
    return bytes(&v, sizeof(T));
  }
  bool str(std::string& s) {
    uint64_t n;
    if (!get(n) || n > size_ - pos_ || n > (1ull << 30)) return false;
    s.resize((size_t)n);
    return bytes(&s[0], n);
  }
  uint64_t left() const { return size_ - pos_; }

 private:
  FILE* f_;
  uint64_t size_, pos_ = 0;
};

// Walk past one value of type t without keeping it (the elements of nested
// arrays, which the reader lists but does not store).
bool skip_value(Reader& r, uint32_t t, int depth) {
  if (depth > 8) return false;
  if (t == GV_STRING) {
    uint64_t n;
    return r.get(n) && r.skip(n);
  }
  if (t == GV_ARRAY) {
    uint32_t et;
    uint64_t n;
    if (!r.get(et) || !r.get(n)) return false;
    const uint64_t eb = scalar_bytes(et);
    if (eb) return n <= r.left() / eb && r.skip(n * eb);
    if (et != GV_STRING && et != GV_ARRAY) return false;
    if (n > r.left() / 8) return false;  // every element takes at least a length or count word
    for (uint64_t k = 0; k < n; ++k)
      if (!skip_value(r, et, depth + 1)) return false;
    return true;
  }
  const uint64_t b = scalar_bytes(t);
  return b && r.skip(b);
}

bool read_value(Reader& r, Meta& m) {
  if (m.type == GV_STRING) {
    m.strs.resize(1);
    return r.str(m.strs[0]);
  }
  if (m.type == GV_ARRAY) {
    if (!r.get(m.elem_type) || !r.get(m.count)) return false;
    if (m.elem_type == GV_ARRAY) {  // listed with its count; the elements are skipped
      if (m.count > r.left() / 12) return false;
      for (uint64_t k = 0; k < m.count; ++k)
        if (!skip_value(r, GV_ARRAY, 1)) return false;
      return true;
    }
    if (m.elem_type == GV_STRING) {
      if (m.count > r.left() / 8) return false;  // every string takes at least its length word
      m.strs.resize((size_t)m.count);
      for (auto& s : m.strs)
        if (!r.str(s)) return false;
      return true;
    }
    const uint64_t eb = scalar_bytes(m.elem_type);
    if (!eb || m.count > r.left() / eb) return false;
    m.data.resize((size_t)(m.count * eb));
    return r.bytes(m.data.data(), m.count * eb);
  }
  const uint64_t b = scalar_bytes(m.type);
  if (!b) return false;
  m.data.resize((size_t)b);
  return r.bytes(m.data.data(), b);
}

void set_err(char* err, size_t len, const char* msg, const std::string& what = "") {
  if (err && len) snprintf(err, len, "%s%s%s", msg, what.empty() ? "" : ": ", what.c_str());
}

}  // namespace

namespace kq {
int api_fail(kq_ctx* ctx, int status, const char* msg);
}

struct kq_gguf {
  std::string path;
  uint32_t version = 0;
  uint64_t alignment = 32, data_start = 0, file_size = 0;
  std::vector<Meta> meta;
  std::vector<Tensor> tensors;
};

extern "C" {

int kq_gguf_open(const char* path, kq_gguf** out, char* err, size_t err_len) {
  if (err && err_len) err[0] = 0;
  if (!path || !out) {
    set_err(err, err_len, "path and out must not be null");
    return KQ_ERR_INVALID_ARG;
  }
  *out = nullptr;
  FILE* f = fopen(path, "rb");
  if (!f) {
    set_err(err, err_len, "cannot open", path);
    return KQ_ERR_FORMAT;
  }
  int rc = KQ_ERR_FORMAT;
  kq_gguf* g = new kq_gguf();
  g->path = path;
  do {
    if (fseeko(f, 0, SEEK_END) != 0) break;
    const off_t end = ftello(f);
    if (end < 0 || fseeko(f, 0, SEEK_SET) != 0) break;
    g->file_size = (uint64_t)end;
    Reader r(f, g->file_size);
    uint32_t magic = 0;
    uint64_t nt = 0, nkv = 0;
    if (!r.get(magic) || magic != 0x46554747u) {
      set_err(err, err_len, "not a GGUF file (bad magic)", path);
      break;
    }
    if (!r.get(g->version) || (g->version != 2 && g->version != 3)) {
      set_err(err, err_len, "unsupported GGUF version (2 and 3 are read)", path);
      break;
    }
    if (!r.get(nt) || !r.get(nkv) || nt > (1u << 24) || nkv > (1u << 24)) {
      set_err(err, err_len, "implausible tensor or metadata count", path);
      break;
    }
    bool ok = true;
    g->meta.resize((size_t)nkv);
    for (auto& m : g->meta) {
      if (!r.str(m.key) || !r.get(m.type) || !read_value(r, m)) {
        ok = false;
        set_err(err, err_len, "truncated or malformed metadata", m.key);
        break;
      }
      if (m.key == "general.alignment" && m.type == GV_U32) {
        uint32_t a;
        memcpy(&a, m.data.data(), 4);
        if (a == 0 || (a & (a - 1))) {
          ok = false;
          set_err(err, err_len, "general.alignment is not a power of two", path);
          break;
        }
        g->alignment = a;
      }
    }
    if (!ok) break;
    g->tensors.resize((size_t)nt);
    for (auto& t : g->tensors) {
      if (!r.str(t.name) || !r.get(t.n_dims) || t.n_dims < 1 || t.n_dims > 4) {
        ok = false;
        set_err(err, err_len, "truncated or malformed tensor entry", t.name);
        break;
      }
      for (uint32_t d = 0; d < t.n_dims && ok; ++d) {
        uint64_t v;
        ok = r.get(v) && v <= (1ull << 40);
        t.ne[d] = (int64_t)v;
      }
      if (!ok || !r.get(t.type) || !r.get(t.offset)) {
        ok = false;
        set_err(err, err_len, "truncated or malformed tensor entry", t.name);
        break;
      }
    }
    if (!ok) break;
    {
      // a tensor name identifies one tensor: a directory that repeats a name is malformed
      std::set<std::string> seen;
      for (const auto& t : g->tensors)
        if (!seen.insert(t.name).second) {
          ok = false;
          set_err(err, err_len, "tensor name appears twice in the directory", t.name);
          break;
        }
    }
    if (!ok) break;
    g->data_start = (r.pos() + g->alignment - 1) / g->alignment * g->alignment;
    for (auto& t : g->tensors) {
      uint64_t be, bb;
      ggml_block(t.type, be, bb);
      if (be) {
        if (t.ne[0] % (int64_t)be) {
          ok = false;
          set_err(err, err_len, "row length is not a whole number of blocks", t.name);
          break;
        }
        unsigned __int128 n = (unsigned __int128)((uint64_t)t.ne[0] / be) * bb;
        for (uint32_t d = 1; d < t.n_dims && n <= g->file_size; ++d) n *= (uint64_t)t.ne[d];
        t.nbytes = n > g->file_size ? g->file_size + 1 : (uint64_t)n;  // too large: fails the bound below
      }
      if (t.offset % g->alignment || t.offset > g->file_size || g->data_start > g->file_size - t.offset ||
          t.nbytes > g->file_size - g->data_start - t.offset) {
        ok = false;
        set_err(err, err_len, "tensor data lies outside the file", t.name);
        break;
      }
      t.offset += g->data_start;
    }
    if (!ok) break;
    rc = KQ_OK;
  } while (false);
  fclose(f);
  if (rc != KQ_OK) {
    if (err && err_len && !err[0]) set_err(err, err_len, "truncated or unreadable GGUF file", path);
    delete g;
    return rc;
  }
  *out = g;
  return KQ_OK;
}

void kq_gguf_close(kq_gguf* f) { delete f; }

int64_t kq_gguf_tensor_count(const kq_gguf* f) { return f ? (int64_t)f->tensors.size() : -1; }

int64_t kq_gguf_find_tensor(const kq_gguf* f, const char* name) {
  if (!f || !name) return -1;
  for (size_t i = 0; i < f->tensors.size(); ++i)
    if (f->tensors[i].name == name) return (int64_t)i;
  return -1;
}

int kq_gguf_tensor_info(const kq_gguf* f, int64_t i, const char** name, int* ggml_type, int* n_dims, int64_t* dims,
                        uint64_t* file_offset, uint64_t* nbytes) {
  if (!f || i < 0 || i >= (int64_t)f->tensors.size()) return KQ_ERR_INVALID_ARG;
  const Tensor& t = f->tensors[(size_t)i];
  if (name) *name = t.name.c_str();
  if (ggml_type) *ggml_type = (int)t.type;
  if (n_dims) *n_dims = (int)t.n_dims;
  if (dims)
    for (int d = 0; d < 4; ++d) dims[d] = t.ne[d];
  if (file_offset) *file_offset = t.offset;
  if (nbytes) *nbytes = t.nbytes;
  return KQ_OK;
}

int kq_gguf_read_tensor(const kq_gguf* f, int64_t i, void* dst, uint64_t dst_bytes) {
  if (!f || i < 0 || i >= (int64_t)f->tensors.size() || (!dst && dst_bytes)) return KQ_ERR_INVALID_ARG;
  const Tensor& t = f->tensors[(size_t)i];
  if (!t.nbytes && t.ne[0]) return KQ_ERR_UNSUPPORTED;  // a type the reader does not size
  if (dst_bytes < t.nbytes) return KQ_ERR_SHORT_BUFFER;
  FILE* fp = fopen(f->path.c_str(), "rb");
  if (!fp) return KQ_ERR_FORMAT;
  const bool ok = fseeko(fp, (off_t)t.offset, SEEK_SET) == 0 &&
                  (t.nbytes == 0 || fread(dst, 1, (size_t)t.nbytes, fp) == (size_t)t.nbytes);
  fclose(fp);
  return ok ? KQ_OK : KQ_ERR_FORMAT;
}

int kq_gguf_upload(kq_ctx* ctx, const kq_gguf* f, int64_t i, kq_weight** out) {
  if (!ctx) return KQ_ERR_INVALID_ARG;
  if (!out || !f || i < 0 || i >= (int64_t)f->tensors.size())
    return kq::api_fail(ctx, KQ_ERR_INVALID_ARG, "kq_gguf_upload: null argument or tensor index out of range");
  *out = nullptr;
  const Tensor& t = f->tensors[(size_t)i];
  if ((t.type != KQ_GGUF_Q2_K && t.type != KQ_GGUF_Q3_K && t.type != KQ_GGUF_Q4_K && t.type != KQ_GGUF_Q5_K &&
       t.type != KQ_GGUF_Q6_K) ||
      t.n_dims != 2)
    return kq::api_fail(ctx, KQ_ERR_UNSUPPORTED,
                        ("kq_gguf_upload: " + t.name + " is not a 2-D Q2_K / Q3_K / Q4_K / Q5_K / Q6_K tensor").c_str());
  void* host = malloc(t.nbytes ? (size_t)t.nbytes : 1);
  if (!host) return kq::api_fail(ctx, KQ_ERR_NOMEM, "kq_gguf_upload: no host memory for the tensor bytes");
  int rc = kq_gguf_read_tensor(f, i, host, t.nbytes);
  if (rc != KQ_OK) kq::api_fail(ctx, rc, ("kq_gguf_upload: cannot read " + t.name).c_str());
  // ne[0] = in_features (the row), ne[1] = out_features (rows)
  if (rc == KQ_OK) rc = kq_weight_upload(ctx, (int)t.type, host, (size_t)t.nbytes, t.ne[1], t.ne[0], out);
  free(host);
  return rc;
}

int64_t kq_gguf_meta_count(const kq_gguf* f) { return f ? (int64_t)f->meta.size() : -1; }

int64_t kq_gguf_find_meta(const kq_gguf* f, const char* key) {
  if (!f || !key) return -1;
  for (size_t i = 0; i < f->meta.size(); ++i)
    if (f->meta[i].key == key) return (int64_t)i;
  return -1;
}

int kq_gguf_meta_info(const kq_gguf* f, int64_t i, const char** key, int* value_type, int* elem_type,
                      uint64_t* count) {
  if (!f || i < 0 || i >= (int64_t)f->meta.size()) return KQ_ERR_INVALID_ARG;
  const Meta& m = f->meta[(size_t)i];
  if (key) *key = m.key.c_str();
  if (value_type) *value_type = (int)m.type;
  if (elem_type) *elem_type = m.type == GV_ARRAY ? (int)m.elem_type : -1;
  if (count) *count = m.count;
  return KQ_OK;
}

int kq_gguf_meta_int(const kq_gguf* f, int64_t i, int64_t* v) {
  if (!f || !v || i < 0 || i >= (int64_t)f->meta.size()) return KQ_ERR_INVALID_ARG;
  const Meta& m = f->meta[(size_t)i];
  const uint8_t* p = m.data.data();
  switch (m.type) {
    case GV_U8: case GV_BOOL: *v = p[0]; return KQ_OK;
    case GV_I8: *v = (int8_t)p[0]; return KQ_OK;
    case GV_U16: { uint16_t x; memcpy(&x, p, 2); *v = x; return KQ_OK; }
    case GV_I16: { int16_t x; memcpy(&x, p, 2); *v = x; return KQ_OK; }
    case GV_U32: { uint32_t x; memcpy(&x, p, 4); *v = x; return KQ_OK; }
    case GV_I32: { int32_t x; memcpy(&x, p, 4); *v = x; return KQ_OK; }
    case GV_U64: { uint64_t x; memcpy(&x, p, 8); if (x > (uint64_t)INT64_MAX) return KQ_ERR_UNSUPPORTED; *v = (int64_t)x; return KQ_OK; }
    case GV_I64: { int64_t x; memcpy(&x, p, 8); *v = x; return KQ_OK; }
    default: return KQ_ERR_UNSUPPORTED;
  }
}

int kq_gguf_meta_float(const kq_gguf* f, int64_t i, double* v) {
  if (!f || !v || i < 0 || i >= (int64_t)f->meta.size()) return KQ_ERR_INVALID_ARG;
  const Meta& m = f->meta[(size_t)i];
  if (m.type == GV_F32) {
    float x;
    memcpy(&x, m.data.data(), 4);
    *v = x;
    return KQ_OK;
  }
  if (m.type == GV_F64) {
    memcpy(v, m.data.data(), 8);
    return KQ_OK;
  }
  int64_t iv;
  const int rc = kq_gguf_meta_int(f, i, &iv);
  if (rc == KQ_OK) *v = (double)iv;
  return rc;
}

int kq_gguf_meta_string(const kq_gguf* f, int64_t i, uint64_t j, const char** s, uint64_t* len) {
  if (!f || !s || i < 0 || i >= (int64_t)f->meta.size()) return KQ_ERR_INVALID_ARG;
  const Meta& m = f->meta[(size_t)i];
  const bool is_str = m.type == GV_STRING || (m.type == GV_ARRAY && m.elem_type == GV_STRING);
  if (!is_str) return KQ_ERR_UNSUPPORTED;
  if (j >= m.strs.size()) return KQ_ERR_INVALID_ARG;
  *s = m.strs[(size_t)j].c_str();
  if (len) *len = m.strs[(size_t)j].size();
  return KQ_OK;
}

int kq_gguf_meta_array(const kq_gguf* f, int64_t i, const void** data, uint64_t* elem_bytes) {
  if (!f || !data || i < 0 || i >= (int64_t)f->meta.size()) return KQ_ERR_INVALID_ARG;
  const Meta& m = f->meta[(size_t)i];
  if (m.type != GV_ARRAY || m.elem_type == GV_STRING) return KQ_ERR_UNSUPPORTED;
  *data = m.data.data();
  if (elem_bytes) *elem_bytes = scalar_bytes(m.elem_type);
  return KQ_OK;
}

}  // extern "C"
