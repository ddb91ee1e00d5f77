// GGUF files on the host: a reader that maps the file in place (with a
// readable zero tail after it) and a writer, behind the tnn_gguf_* calls toy's
// loaders and its checkpoint writer make (tinynn/tinynn_gguf.h,
// tinynn/tinynn_ggml.h:538-545); plus the step engine's bridge: load a model's
// tensors from a GGUF (Q8_0 blocks verbatim into the frozen-base arena, f32
// into the parameter arenas, Adam moments from "<name>.m" / "<name>.v"), and
// save trainable tensors (and moments) as a checkpoint.
//
// Format (GGUF v3, little endian): "GGUF", version u32, tensor count u64, kv
// count u64; kv pairs (key string, value type u32, value); tensor infos (name
// string, n_dims u32, ne[n_dims] u64 with ne0 the fastest, ggml type u32,
// data offset u64 relative to the data section); the data section starts at
// the next multiple of general.alignment (32 when absent) and every tensor's
// data is aligned to it. A string is a u64 length and its bytes.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include <cuda_fp16.h>

#include "session.cuh"
#include "toy_b200.h"

namespace {

enum : uint32_t {
  kU8 = 0, kI8, kU16, kI16, kU32, kI32, kF32, kBool, kStr, kArr, kU64, kI64, kF64
};
enum : int { kTypeF32 = 0, kTypeF16 = 1, kTypeQ8_0 = 8, kTypeBF16 = 30 };

struct KV {
  std::string key;
  uint32_t type = 0;
  uint64_t u = 0;     // integer / bool payload
  int64_t i = 0;
  double f = 0.0;
  std::string s;
  uint32_t arr_type = 0;
  std::vector<std::string> arr_s;
  std::vector<int64_t> arr_i;
  std::vector<double> arr_f;
};

struct TInfo {
  std::string name;
  int n_dims = 0;
  int64_t ne[4] = {1, 1, 1, 1};
  int type = 0;
  uint64_t offset = 0;   // relative to the data section
};

struct Gguf {
  std::vector<KV> kv;
  std::vector<TInfo> t;
  const uint8_t* map = nullptr;   // file bytes, followed by >= TNN_GGUF_MMAP_TAIL zero bytes
  size_t size = 0, map_len = 0;
  uint64_t data_off = 0;
  uint32_t align = 32;
  std::string arch;
};

int64_t type_nbytes(int type, int64_t nel) {
  switch (type) {
    case kTypeF32: return nel * 4;
    case kTypeF16:
    case kTypeBF16: return nel * 2;
    case kTypeQ8_0: return nel % 32 ? -1 : nel / 32 * 34;
    default: return -1;
  }
}

struct Reader {
  const uint8_t* p;
  size_t n, pos = 0;
  bool ok = true;
  bool get(void* dst, size_t k) {
    if (!ok || pos + k > n) return ok = false;
    memcpy(dst, p + pos, k);
    pos += k;
    return true;
  }
  template <class T>
  T v() {
    T x{};
    get(&x, sizeof(T));
    return x;
  }
  std::string str() {
    const uint64_t len = v<uint64_t>();
    if (!ok || len > n - pos) {
      ok = false;
      return std::string();
    }
    std::string s(reinterpret_cast<const char*>(p + pos), (size_t)len);
    pos += (size_t)len;
    return s;
  }
};

bool read_scalar(Reader& r, uint32_t type, KV& kv) {
  switch (type) {
    case kU8: kv.u = r.v<uint8_t>(); kv.i = (int64_t)kv.u; kv.f = (double)kv.u; break;
    case kI8: kv.i = r.v<int8_t>(); kv.u = (uint64_t)kv.i; kv.f = (double)kv.i; break;
    case kU16: kv.u = r.v<uint16_t>(); kv.i = (int64_t)kv.u; kv.f = (double)kv.u; break;
    case kI16: kv.i = r.v<int16_t>(); kv.u = (uint64_t)kv.i; kv.f = (double)kv.i; break;
    case kU32: kv.u = r.v<uint32_t>(); kv.i = (int64_t)kv.u; kv.f = (double)kv.u; break;
    case kI32: kv.i = r.v<int32_t>(); kv.u = (uint64_t)kv.i; kv.f = (double)kv.i; break;
    case kU64: kv.u = r.v<uint64_t>(); kv.i = (int64_t)kv.u; kv.f = (double)kv.u; break;
    case kI64: kv.i = r.v<int64_t>(); kv.u = (uint64_t)kv.i; kv.f = (double)kv.i; break;
    case kF32: kv.f = r.v<float>(); break;
    case kF64: kv.f = r.v<double>(); break;
    case kBool: kv.u = r.v<uint8_t>(); kv.i = (int64_t)kv.u; break;
    case kStr: kv.s = r.str(); break;
    default: return false;
  }
  return r.ok;
}

bool parse(Gguf& g) {
  Reader r{g.map, g.size};
  if (r.v<uint32_t>() != 0x46554747u) return false;   // "GGUF"
  const uint32_t version = r.v<uint32_t>();
  if (version < 2 || version > 3) return false;
  const uint64_t nt = r.v<uint64_t>(), nkv = r.v<uint64_t>();
  if (!r.ok || nt > (1u << 24) || nkv > (1u << 24)) return false;
  g.kv.resize((size_t)nkv);
  for (auto& kv : g.kv) {
    kv.key = r.str();
    kv.type = r.v<uint32_t>();
    if (kv.type == kArr) {
      kv.arr_type = r.v<uint32_t>();
      const uint64_t n = r.v<uint64_t>();
      if (!r.ok || n > r.n) return false;
      for (uint64_t j = 0; j < n; ++j) {
        KV e;
        if (!read_scalar(r, kv.arr_type, e)) return false;
        if (kv.arr_type == kStr) kv.arr_s.push_back(std::move(e.s));
        else if (kv.arr_type == kF32 || kv.arr_type == kF64) kv.arr_f.push_back(e.f);
        else kv.arr_i.push_back(e.i);
      }
    } else if (!read_scalar(r, kv.type, kv)) {
      return false;
    }
    if (kv.key == "general.alignment" && (kv.type == kU32 || kv.type == kI32) && kv.u > 0) g.align = (uint32_t)kv.u;
    if (kv.key == "general.architecture" && kv.type == kStr) g.arch = kv.s;
  }
  g.t.resize((size_t)nt);
  for (auto& t : g.t) {
    t.name = r.str();
    t.n_dims = (int)r.v<uint32_t>();
    if (!r.ok || t.n_dims < 1 || t.n_dims > 4) return false;
    for (int d = 0; d < t.n_dims; ++d) t.ne[d] = (int64_t)r.v<uint64_t>();
    t.type = (int)r.v<uint32_t>();
    t.offset = r.v<uint64_t>();
  }
  if (!r.ok || g.align == 0) return false;
  g.data_off = (r.pos + g.align - 1) / g.align * g.align;
  for (const auto& t : g.t) {
    const int64_t nb = type_nbytes(t.type, t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3]);
    if (nb >= 0 && g.data_off + t.offset + (uint64_t)nb > g.size) return false;
  }
  return true;
}

Gguf* G(void* h) { return static_cast<Gguf*>(h); }

const KV* find_kv(const Gguf* g, const char* key) {
  if (!g || !key) return nullptr;
  for (const auto& kv : g->kv)
    if (kv.key == key) return &kv;
  return nullptr;
}

// ---------------------------------------------------------------- writer
struct WTensor {
  std::string name;
  int n_dims = 2;
  int64_t ne[4] = {1, 1, 1, 1};
  int type = kTypeF32;
  std::vector<uint8_t> data;
};

struct Writer {
  std::vector<KV> kv;
  std::vector<WTensor> t;
};

void put_kv(Writer* w, const char* key, KV kv) {
  if (!w || !key) return;
  kv.key = key;
  for (auto& e : w->kv)
    if (e.key == kv.key) {
      e = kv;
      return;
    }
  w->kv.push_back(kv);
}

void wr(std::vector<uint8_t>& b, const void* p, size_t n) {
  const uint8_t* c = static_cast<const uint8_t*>(p);
  b.insert(b.end(), c, c + n);
}
template <class T>
void wv(std::vector<uint8_t>& b, T x) {
  wr(b, &x, sizeof(T));
}
void ws(std::vector<uint8_t>& b, const std::string& s) {
  wv<uint64_t>(b, s.size());
  wr(b, s.data(), s.size());
}

float half_bits_to_float(uint16_t h) {
  __half_raw r;
  r.x = h;
  return __half2float(__half(r));
}

int to_f32(const Gguf* g, int i, std::vector<float>& out) {
  const TInfo& t = g->t[i];
  const int64_t nel = t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3];
  const uint8_t* src = g->map + g->data_off + t.offset;
  out.resize((size_t)nel);
  switch (t.type) {
    case kTypeF32: memcpy(out.data(), src, (size_t)nel * 4); return 0;
    case kTypeF16:
      for (int64_t k = 0; k < nel; ++k) {
        uint16_t h;
        memcpy(&h, src + 2 * k, 2);
        out[k] = half_bits_to_float(h);
      }
      return 0;
    case kTypeBF16:
      for (int64_t k = 0; k < nel; ++k) {
        uint16_t h;
        memcpy(&h, src + 2 * k, 2);
        const uint32_t u = (uint32_t)h << 16;
        memcpy(&out[k], &u, 4);
      }
      return 0;
    case kTypeQ8_0:
      if (nel % 32) return -1;
      for (int64_t b = 0; b < nel / 32; ++b) {
        const uint8_t* q = src + b * 34;
        const float d = half_bits_to_float((uint16_t)(q[0] | (q[1] << 8)));
        for (int j = 0; j < 32; ++j) out[b * 32 + j] = d * (float)(int8_t)q[2 + j];
      }
      return 0;
    default: return -1;
  }
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------- reader
void* tnn_gguf_load(const char* path) {
  if (!path) return nullptr;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return nullptr;
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size <= 0) {
    close(fd);
    return nullptr;
  }
  const size_t fsize = (size_t)st.st_size;
  const size_t page = (size_t)sysconf(_SC_PAGESIZE);
  const size_t map_len = (fsize + page - 1) / page * page + TNN_GGUF_MMAP_TAIL;
  // anonymous zero pages with the file mapped over the front: the bytes past
  // EOF up to the page boundary are zero, the tail pages after it too
  void* resv = mmap(nullptr, map_len, PROT_READ, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
  if (resv == MAP_FAILED) {
    close(fd);
    return nullptr;
  }
  void* m = mmap(resv, fsize, PROT_READ, MAP_PRIVATE | MAP_FIXED, fd, 0);
  close(fd);
  if (m == MAP_FAILED) {
    munmap(resv, map_len);
    return nullptr;
  }
  auto g = std::make_unique<Gguf>();
  g->map = static_cast<const uint8_t*>(m);
  g->size = fsize;
  g->map_len = map_len;
  if (!parse(*g)) {
    munmap(resv, map_len);
    return nullptr;
  }
  return g.release();
}

void tnn_gguf_free(void* handle) {
  Gguf* g = G(handle);
  if (!g) return;
  if (g->map) munmap(const_cast<uint8_t*>(g->map), g->map_len);
  delete g;
}

int tnn_gguf_n_tensors(void* handle) { return handle ? (int)G(handle)->t.size() : -1; }

const char* tnn_gguf_tensor_name(void* handle, int i) {
  Gguf* g = G(handle);
  if (!g || i < 0 || i >= (int)g->t.size()) return nullptr;
  return g->t[i].name.c_str();
}

int tnn_gguf_tensor_ne(void* handle, int i, int dim) {
  Gguf* g = G(handle);
  if (!g || i < 0 || i >= (int)g->t.size() || dim < 0 || dim > 3) return -1;
  return (int)g->t[i].ne[dim];
}

int tnn_gguf_tensor_type(void* handle, int i) {
  Gguf* g = G(handle);
  if (!g || i < 0 || i >= (int)g->t.size()) return -1;
  return g->t[i].type;
}

size_t tnn_gguf_tensor_nbytes(void* handle, int i) {
  Gguf* g = G(handle);
  if (!g || i < 0 || i >= (int)g->t.size()) return 0;
  const TInfo& t = g->t[i];
  const int64_t nb = type_nbytes(t.type, t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3]);
  return nb < 0 ? 0 : (size_t)nb;
}

int tnn_gguf_tensor_is_quantized(void* handle, int i) {
  const int ty = tnn_gguf_tensor_type(handle, i);
  return ty < 0 ? -1 : (ty == kTypeF32 || ty == kTypeF16 || ty == kTypeBF16) ? 0 : 1;
}

int tnn_gguf_find_index(void* handle, const char* name) {
  Gguf* g = G(handle);
  if (!g || !name) return -1;
  for (size_t i = 0; i < g->t.size(); ++i)
    if (g->t[i].name == name) return (int)i;
  return -1;
}

int tnn_gguf_read_f32_to_doubles(void* handle, int i, double* out, size_t n) {
  Gguf* g = G(handle);
  if (!g || !out || i < 0 || i >= (int)g->t.size()) return -1;
  std::vector<float> v;
  if (to_f32(g, i, v)) return -1;
  if (n != v.size()) return -1;
  for (size_t k = 0; k < n; ++k) out[k] = v[k];
  return 0;
}

int tnn_gguf_get_u32(void* handle, const char* key) {
  const KV* kv = find_kv(G(handle), key);
  if (!kv || !(kv->type == kU32 || kv->type == kI32 || kv->type == kU16 || kv->type == kU8 || kv->type == kU64 ||
               kv->type == kI64 || kv->type == kI16 || kv->type == kI8))
    return -1;
  return (int)kv->i;
}

double tnn_gguf_get_f32(void* handle, const char* key) {
  const KV* kv = find_kv(G(handle), key);
  if (!kv || !(kv->type == kF32 || kv->type == kF64)) return 0.0;
  return kv->f;
}

int tnn_gguf_get_bool(void* handle, const char* key) {
  const KV* kv = find_kv(G(handle), key);
  if (!kv || kv->type != kBool) return -1;
  return kv->u ? 1 : 0;
}

const char* tnn_gguf_get_str(void* handle, const char* key) {
  const KV* kv = find_kv(G(handle), key);
  if (!kv || kv->type != kStr) return nullptr;
  return kv->s.c_str();
}

const char* tnn_gguf_arch_prefix(void* handle) {
  Gguf* g = G(handle);
  return g ? g->arch.c_str() : "";
}

int tnn_gguf_arr_n(void* handle, const char* key) {
  const KV* kv = find_kv(G(handle), key);
  if (!kv || kv->type != kArr) return -1;
  return (int)(kv->arr_type == kStr ? kv->arr_s.size()
                                    : (kv->arr_type == kF32 || kv->arr_type == kF64) ? kv->arr_f.size()
                                                                                     : kv->arr_i.size());
}

const char* tnn_gguf_arr_str(void* handle, const char* key, int i) {
  const KV* kv = find_kv(G(handle), key);
  if (!kv || kv->type != kArr || kv->arr_type != kStr || i < 0 || i >= (int)kv->arr_s.size()) return nullptr;
  return kv->arr_s[i].c_str();
}

int tnn_gguf_arr_i32(void* handle, const char* key, int i) {
  const KV* kv = find_kv(G(handle), key);
  if (!kv || kv->type != kArr || kv->arr_type == kStr || kv->arr_type == kF32 || kv->arr_type == kF64 || i < 0 ||
      i >= (int)kv->arr_i.size())
    return -1;
  return (int)kv->arr_i[i];
}

int tnn_gguf_is_native_layout(void* handle) {
  Gguf* g = G(handle);
  if (!g) return 0;
  if (tnn_gguf_get_bool(handle, "toy.ggml_native") == 1) return 1;
  if (g->arch.empty()) return 0;
  const int d = tnn_gguf_get_u32(handle, (g->arch + ".embedding_length").c_str());
  const int ff = tnn_gguf_get_u32(handle, (g->arch + ".feed_forward_length").c_str());
  const int idx = tnn_gguf_find_index(handle, "blk.0.ffn_gate.weight");
  if (idx < 0 || d <= 0 || ff <= 0 || d == ff) return 0;
  return (tnn_gguf_tensor_ne(handle, idx, 0) == d && tnn_gguf_tensor_ne(handle, idx, 1) == ff) ? 1 : 0;
}

void* tnn_gguf_mmap_base(void* handle) { return handle ? const_cast<uint8_t*>(G(handle)->map) : nullptr; }
size_t tnn_gguf_mmap_size(void* handle) { return handle ? G(handle)->size : 0; }

size_t tnn_gguf_tensor_file_offset(void* handle, int i) {
  Gguf* g = G(handle);
  if (!g || i < 0 || i >= (int)g->t.size()) return 0;
  return (size_t)(g->data_off + g->t[i].offset);
}

// ---------------------------------------------------------------- writer
void* tnn_gguf_w_init(void) { return new Writer(); }
void tnn_gguf_w_free(void* ctx) { delete static_cast<Writer*>(ctx); }

void tnn_gguf_w_set_str(void* ctx, const char* key, const char* val) {
  KV kv;
  kv.type = kStr;
  kv.s = val ? val : "";
  put_kv(static_cast<Writer*>(ctx), key, kv);
}
void tnn_gguf_w_set_u32(void* ctx, const char* key, int val) {
  KV kv;
  kv.type = kU32;
  kv.u = (uint32_t)val;
  kv.i = val;
  put_kv(static_cast<Writer*>(ctx), key, kv);
}
void tnn_gguf_w_set_f32(void* ctx, const char* key, double val) {
  KV kv;
  kv.type = kF32;
  kv.f = val;
  put_kv(static_cast<Writer*>(ctx), key, kv);
}
void tnn_gguf_w_set_bool(void* ctx, const char* key, int val) {
  KV kv;
  kv.type = kBool;
  kv.u = val ? 1 : 0;
  put_kv(static_cast<Writer*>(ctx), key, kv);
}

int tb2_gguf_w_add_f32(void* ctx, const char* name, int ne0, int ne1, const float* data) {
  Writer* w = static_cast<Writer*>(ctx);
  if (!w || !name || !data || ne0 < 1 || ne1 < 1) return -1;
  WTensor t;
  t.name = name;
  t.n_dims = ne1 > 1 ? 2 : 1;
  t.ne[0] = ne0;
  t.ne[1] = ne1;
  t.type = kTypeF32;
  t.data.resize((size_t)ne0 * ne1 * 4);
  memcpy(t.data.data(), data, t.data.size());
  w->t.push_back(std::move(t));
  return 0;
}

int tb2_gguf_w_add_q8_0(void* ctx, const char* name, int ne0, int ne1, const void* blocks) {
  Writer* w = static_cast<Writer*>(ctx);
  if (!w || !name || !blocks || ne0 < 32 || ne0 % 32 || ne1 < 1) return -1;
  WTensor t;
  t.name = name;
  t.n_dims = 2;
  t.ne[0] = ne0;
  t.ne[1] = ne1;
  t.type = kTypeQ8_0;
  t.data.resize((size_t)ne0 / 32 * 34 * ne1);
  memcpy(t.data.data(), blocks, t.data.size());
  w->t.push_back(std::move(t));
  return 0;
}

// tinynn_ggml.h:543: a tensor of a session -- a parameter of the step
// program (f32 values, or a frozen projection's Q8_0 blocks verbatim) or an
// f32 node of the primitive graph -- copied to the host now.
void tnn_gguf_w_add_tensor(void* ctx, void* tensor) {
  Writer* w = static_cast<Writer*>(ctx);
  tb2::Tensor* t = static_cast<tb2::Tensor*>(tensor);
  if (!w || !t || !t->sess) return;
  tb2::Session* s = t->sess;
  const int ne0 = t->ne[0], ne1 = (int)(t->nel() / t->ne[0]);
  if (t->role == tb2::Tensor::kParam && s->eng) {
    const tb2::Param* p = s->eng->find(t->param);
    if (!p) return;
    if (p->q8) {
      std::vector<uint8_t> b((size_t)p->numel() / 32 * 34);
      if (s->eng->get_param_q8(p->name, b.data(), (long long)b.size()) == 0)
        tb2_gguf_w_add_q8_0(ctx, t->name.c_str(), ne0, ne1, b.data());
    } else {
      std::vector<float> v((size_t)p->numel());
      if (s->eng->get_param(p->name, v.data(), p->numel()) == 0) tb2_gguf_w_add_f32(ctx, t->name.c_str(), ne0, ne1, v.data());
    }
    return;
  }
  if (t->role == tb2::Tensor::kPrim && t->type == kTypeF32 && t->data) {
    std::vector<float> v((size_t)t->nel());
    cudaSetDevice(s->device);
    if (cudaDeviceSynchronize() != cudaSuccess) return;
    const uint8_t* src = static_cast<const uint8_t*>(t->view_of ? t->view_of->data : t->data) + t->view_off;
    if (cudaMemcpy(v.data(), src, v.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess)
      tb2_gguf_w_add_f32(ctx, t->name.c_str(), ne0, ne1, v.data());
  }
}

int tnn_gguf_w_finalize(void* ctx, const char* path) {
  Writer* w = static_cast<Writer*>(ctx);
  if (!w || !path) return -1;
  const uint32_t align = 32;
  std::vector<uint8_t> h;
  wv<uint32_t>(h, 0x46554747u);
  wv<uint32_t>(h, 3);
  wv<uint64_t>(h, w->t.size());
  wv<uint64_t>(h, w->kv.size());
  for (const auto& kv : w->kv) {
    ws(h, kv.key);
    wv<uint32_t>(h, kv.type);
    switch (kv.type) {
      case kStr: ws(h, kv.s); break;
      case kU32: wv<uint32_t>(h, (uint32_t)kv.u); break;
      case kF32: wv<float>(h, (float)kv.f); break;
      case kBool: wv<uint8_t>(h, kv.u ? 1 : 0); break;
      default: return -1;
    }
  }
  uint64_t off = 0;
  std::vector<uint64_t> offs;
  for (const auto& t : w->t) {
    ws(h, t.name);
    wv<uint32_t>(h, (uint32_t)t.n_dims);
    for (int d = 0; d < t.n_dims; ++d) wv<uint64_t>(h, (uint64_t)t.ne[d]);
    wv<uint32_t>(h, (uint32_t)t.type);
    wv<uint64_t>(h, off);
    offs.push_back(off);
    off += (t.data.size() + align - 1) / align * align;
  }
  h.resize((h.size() + align - 1) / align * align, 0);
  FILE* f = fopen(path, "wb");
  if (!f) return -1;
  bool ok = fwrite(h.data(), 1, h.size(), f) == h.size();
  static const uint8_t zeros[32] = {0};
  for (size_t i = 0; ok && i < w->t.size(); ++i) {
    const auto& d = w->t[i].data;
    ok = fwrite(d.data(), 1, d.size(), f) == d.size();
    const size_t pad = (d.size() + align - 1) / align * align - d.size();
    if (ok && pad) ok = fwrite(zeros, 1, pad, f) == pad;
  }
  ok = (fclose(f) == 0) && ok;
  return ok ? 0 : -1;
}

int tnn_gguf_write_demo_file(const char* path) {
  void* w = tnn_gguf_w_init();
  tnn_gguf_w_set_str(w, "general.architecture", "demo");
  const float v[6] = {1, 2, 3, 4, 5, 6};
  tb2_gguf_w_add_f32(w, "demo.tensor", 3, 2, v);
  const int rc = tnn_gguf_w_finalize(w, path);
  tnn_gguf_w_free(w);
  return rc;
}

}  // extern "C"

// ---------------------------------------------------------------- step engine bridge
namespace {

// The per-head LoRA-Q tensors under toy's names (blk.N.attn_q.head_H.lora_{a,b}.weight,
// transformer_block.rb:522-579): head h of the stacked A is rows h r .. (h + 1) r,
// of the stacked B rows h d_head .. (h + 1) d_head.
bool per_head_name(const std::string& packed, int h, std::string& out) {
  const std::string q = ".attn_q.lora_";
  const size_t at = packed.find(q);
  if (at == std::string::npos) return false;
  out = packed.substr(0, at) + ".attn_q.head_" + std::to_string(h) + ".lora_" + packed.substr(at + q.size()) +
        ".weight";
  return true;
}

}  // namespace

extern "C" {

int tb2_llama_load_gguf(void* sess, void* gguf, int flags) {
  if (!sess || !gguf) return -1;
  tb2::Session* s = static_cast<tb2::Session*>(sess);
  Gguf* g = G(gguf);
  if (!s->eng) return -2;
  tb2::LlamaEngine& e = *s->eng;
  const tb2::LlamaConfig& c = e.cfg();
  const bool native = tnn_gguf_is_native_layout(gguf) == 1 || tnn_gguf_find_index(gguf, "blk.0.ffn_gate.weight") < 0;
  int loaded = 0;
  std::vector<float> v;
  for (const tb2::Param& p : e.params()) {
    int i = tnn_gguf_find_index(gguf, p.name.c_str());
    const bool lora = p.name.find(".lora_") != std::string::npos;
    const bool per_head = lora && c.lora_per_head_q && p.name.find(".attn_q.") != std::string::npos;
    if (i < 0 && per_head) {   // toy's per-head names: assemble the stacked tensor
      const int H = c.n_heads, part = (int)(p.numel() / H);
      std::vector<float> full((size_t)p.numel());
      bool all = true;
      for (int h = 0; h < H && all; ++h) {
        std::string nm;
        per_head_name(p.name, h, nm);
        const int j = tnn_gguf_find_index(gguf, nm.c_str());
        if (j < 0 || to_f32(g, j, v) || (int64_t)v.size() != part) {
          all = false;
          break;
        }
        memcpy(full.data() + (size_t)h * part, v.data(), (size_t)part * 4);
      }
      if (all) {
        if (e.set_param(p.name, full.data(), p.numel())) return -3;
        ++loaded;
        continue;
      }
    }
    if (i < 0) {
      // adapters absent from a base model keep their init; a partial file
      // (a checkpoint) leaves every absent tensor as it is
      if (lora || (flags & 2)) continue;
      fprintf(stderr, "[toy_b200] tb2_llama_load_gguf: tensor %s missing from the file\n", p.name.c_str());
      return -1;
    }
    const TInfo& t = g->t[i];
    // toy's legacy layout stores the blocks' 2-D linears transposed (ne=[out, in])
    const bool transposed = !native && p.rows > 1 && p.name.compare(0, 4, "blk.") == 0;
    const int64_t want0 = transposed ? p.rows : p.cols, want1 = transposed ? p.cols : p.rows;
    if (t.ne[0] != want0 || t.ne[1] * t.ne[2] * t.ne[3] != want1) {
      fprintf(stderr, "[toy_b200] tb2_llama_load_gguf: %s has shape [%lld, %lld], expected ne=[%lld, %lld]\n",
              p.name.c_str(), (long long)t.ne[0], (long long)t.ne[1], (long long)want0, (long long)want1);
      return -1;
    }
    if (p.q8 && t.type == kTypeQ8_0 && !transposed) {   // the blocks as they are on disk
      const uint8_t* src = g->map + g->data_off + t.offset;
      if (e.set_param_q8(p.name, src, p.numel() / 32 * 34)) return -3;
      ++loaded;
      continue;
    }
    if (to_f32(g, i, v)) {
      fprintf(stderr, "[toy_b200] tb2_llama_load_gguf: %s has an unsupported type %d\n", p.name.c_str(), t.type);
      return -1;
    }
    if (transposed) {
      std::vector<float> tr(v.size());
      for (int r = 0; r < p.rows; ++r)
        for (int k = 0; k < p.cols; ++k) tr[(size_t)r * p.cols + k] = v[(size_t)k * p.rows + r];
      v.swap(tr);
    }
    if (e.set_param(p.name, v.data(), p.numel())) return -3;
    ++loaded;
  }
  if (flags & 1) {   // Adam moments of the trainable tensors, when the file has them
    for (const tb2::Param& p : e.params()) {
      if (!p.trainable) continue;
      for (int which = 0; which < 2; ++which) {
        const std::string nm = p.name + (which ? ".v" : ".m");
        const int i = tnn_gguf_find_index(gguf, nm.c_str());
        if (i < 0) continue;
        if (to_f32(g, i, v) || (int64_t)v.size() != p.numel()) return -1;
        if (e.set_moment(p.name, which, v.data(), p.numel())) return -3;
        ++loaded;
      }
    }
  }
  return loaded;
}

int tb2_llama_save_gguf(void* sess, const char* path, int what) {
  if (!sess || !path) return -1;
  tb2::Session* s = static_cast<tb2::Session*>(sess);
  if (!s->eng) return -2;
  tb2::LlamaEngine& e = *s->eng;
  const tb2::LlamaConfig& c = e.cfg();
  void* w = tnn_gguf_w_init();
  // the metadata toy's checkpoint writer records (lib/toy/train/toy_gguf_writer.rb)
  tnn_gguf_w_set_str(w, "general.architecture", "llama");
  tnn_gguf_w_set_str(w, "general.name", c.mode == 0 ? "toy-from-scratch" : "toy-lora");
  tnn_gguf_w_set_u32(w, "llama.vocab_size", c.vocab);
  tnn_gguf_w_set_u32(w, "llama.embedding_length", c.d_model);
  tnn_gguf_w_set_u32(w, "llama.feed_forward_length", c.d_ff);
  tnn_gguf_w_set_u32(w, "llama.block_count", c.n_layers);
  tnn_gguf_w_set_u32(w, "llama.attention.head_count", c.n_heads);
  tnn_gguf_w_set_u32(w, "llama.attention.head_count_kv", c.n_kv);
  tnn_gguf_w_set_u32(w, "llama.context_length", c.T);
  tnn_gguf_w_set_f32(w, "llama.attention.layer_norm_rms_epsilon", c.rms_eps);
  tnn_gguf_w_set_f32(w, "llama.rope.freq_base", c.rope_base);
  tnn_gguf_w_set_bool(w, "toy.ggml_native", 1);
  std::vector<float> v;
  int rc = 0;
  for (const tb2::Param& p : e.params()) {
    if (!p.trainable && !(what & 2)) continue;
    if (p.q8) {
      std::vector<uint8_t> b((size_t)p.numel() / 32 * 34);
      if ((rc = e.get_param_q8(p.name, b.data(), (long long)b.size()))) break;
      tb2_gguf_w_add_q8_0(w, p.name.c_str(), p.cols, p.rows, b.data());
      continue;
    }
    v.resize((size_t)p.numel());
    if ((rc = e.get_param(p.name, v.data(), p.numel()))) break;
    const bool per_head = c.lora_per_head_q && p.name.find(".attn_q.lora_") != std::string::npos;
    if (per_head && !(what & 8)) {   // toy's per-head tensors, one pair per query head
      const int H = c.n_heads, rows = p.rows / H;
      for (int h = 0; h < H; ++h) {
        std::string nm;
        per_head_name(p.name, h, nm);
        tb2_gguf_w_add_f32(w, nm.c_str(), p.cols, rows, v.data() + (size_t)h * rows * p.cols);
      }
    } else {
      tb2_gguf_w_add_f32(w, p.name.c_str(), p.cols, p.rows, v.data());
    }
    if ((what & 4) && p.trainable) {
      for (int which = 0; which < 2 && !rc; ++which) {
        std::vector<float> mv((size_t)p.numel());
        if ((rc = e.get_moment(p.name, which, mv.data(), p.numel()))) break;
        tb2_gguf_w_add_f32(w, (p.name + (which ? ".v" : ".m")).c_str(), p.cols, p.rows, mv.data());
      }
      if (rc) break;
    }
  }
  if (!rc) rc = tnn_gguf_w_finalize(w, path);
  tnn_gguf_w_free(w);
  return rc;
}

}  // extern "C"
