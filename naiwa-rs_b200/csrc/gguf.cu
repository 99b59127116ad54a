// gguf.cu — on-disk GGUF expert stacks into moe_layer_desc (include/moe_b200.h, moe_gguf_*).
//
// The reference loads its model from GGUF shards through candle (src/load.rs:414-450 checks the
// header, the architecture and that every tensor's type can run) and hands the provider each MoE
// block's stacked expert tensors, blk.{L}.ffn_{gate,up,down}_exps.weight, as [E, N, K] GGML
// QTensors (provider.rs:367, expert_qtensors), which it slices per expert by byte range
// (expert.rs:123-145: stride = N * (K / block) * type_size). This file reads the same files: it
// maps the file read-only, parses the GGUF v2/v3 header, metadata and tensor table with bounds
// checks on every read, and points a moe_layer_desc's host stacks straight into the mapping, so a
// layer is created from the file's own bytes with no copy (the router alone is converted to bf16
// when the file stores it as f32 or f16).
//
// GGUF layout (little endian): "GGUF", u32 version, u64 tensor count, u64 metadata count; metadata
// = (string key, u32 type, value)*; tensor infos = (string name, u32 n_dims, u64 dims[n_dims] with
// dims[0] the fastest, u32 ggml type, u64 offset)*; tensor data starts at the next multiple of
// general.alignment (default 32). Strings are u64 length + bytes.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "moe_internal.cuh"

namespace moe {
namespace {

enum : uint32_t {  // GGUF metadata value types
  GV_U8 = 0, GV_I8 = 1, GV_U16 = 2, GV_I16 = 3, GV_U32 = 4, GV_I32 = 5, GV_F32 = 6, GV_BOOL = 7,
  GV_STRING = 8, GV_ARRAY = 9, GV_U64 = 10, GV_I64 = 11, GV_F64 = 12
};

enum : int {  // GGML tensor types this library reads
  GT_F32 = 0, GT_F16 = 1, GT_Q8_0 = 8, GT_Q4_K = 12, GT_BF16 = 30
};

// (elements per block, bytes per block) of the GGML types whose byte size is known here; 0 = unknown.
void ggml_block(int type, int64_t* block, int64_t* bytes) {
  static const std::map<int, std::pair<int, int>> t = {
      {0, {1, 4}},      {1, {1, 2}},      {2, {32, 18}},    {3, {32, 20}},   {6, {32, 22}},   {7, {32, 24}},
      {8, {32, 34}},    {9, {32, 36}},    {10, {256, 84}},  {11, {256, 110}}, {12, {256, 144}}, {13, {256, 176}},
      {14, {256, 210}}, {15, {256, 292}}, {24, {1, 1}},     {25, {1, 2}},    {26, {1, 4}},    {27, {1, 8}},
      {28, {1, 8}},     {30, {1, 2}}};
  auto it = t.find(type);
  *block = it == t.end() ? 0 : it->second.first;
  *bytes = it == t.end() ? 0 : it->second.second;
}

const char* ggml_type_name(int type) {
  switch (type) {
    case GT_F32: return "F32";
    case GT_F16: return "F16";
    case GT_Q8_0: return "Q8_0";
    case GT_Q4_K: return "Q4_K";
    case GT_BF16: return "BF16";
    default: return "other";
  }
}

struct Value {
  uint32_t type = 0;
  int64_t i = 0;
  double f = 0.0;
  std::string s;
};

struct TensorInfo {
  std::string name;
  int type = 0;
  int n_dims = 0;
  int64_t dims[4] = {1, 1, 1, 1};
  uint64_t offset = 0;
  int64_t nbytes = -1;  // -1: type of unknown size
  const uint8_t* data = nullptr;
};

// Bounds-checked reader over the mapping.
struct Cursor {
  const uint8_t* base;
  size_t size, pos = 0;
  bool ok = true;
  bool need(size_t n) {
    if (!ok || n > size - pos) ok = false;
    return ok;
  }
  template <class T>
  T get() {
    T v{};
    if (need(sizeof(T))) {
      std::memcpy(&v, base + pos, sizeof(T));
      pos += sizeof(T);
    }
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (!ok || n > (uint64_t)1 << 24 || !need((size_t)n)) {
      ok = false;
      return {};
    }
    std::string s(reinterpret_cast<const char*>(base + pos), (size_t)n);
    pos += (size_t)n;
    return s;
  }
  void skip_value(uint32_t type, int depth = 0) {
    switch (type) {
      case GV_U8: case GV_I8: case GV_BOOL: need(1) && (pos += 1); break;
      case GV_U16: case GV_I16: need(2) && (pos += 2); break;
      case GV_U32: case GV_I32: case GV_F32: need(4) && (pos += 4); break;
      case GV_U64: case GV_I64: case GV_F64: need(8) && (pos += 8); break;
      case GV_STRING: (void)str(); break;
      case GV_ARRAY: {
        const uint32_t et = get<uint32_t>();
        const uint64_t n = get<uint64_t>();
        if (depth > 2 || n > size) {
          ok = false;
          break;
        }
        for (uint64_t i = 0; i < n && ok; ++i) skip_value(et, depth + 1);
        break;
      }
      default: ok = false;
    }
  }
  Value value(uint32_t type) {
    Value v;
    v.type = type;
    switch (type) {
      case GV_U8: v.i = get<uint8_t>(); break;
      case GV_I8: v.i = get<int8_t>(); break;
      case GV_U16: v.i = get<uint16_t>(); break;
      case GV_I16: v.i = get<int16_t>(); break;
      case GV_U32: v.i = get<uint32_t>(); break;
      case GV_I32: v.i = get<int32_t>(); break;
      case GV_U64: v.i = (int64_t)get<uint64_t>(); break;
      case GV_I64: v.i = get<int64_t>(); break;
      case GV_BOOL: v.i = get<uint8_t>() != 0; break;
      case GV_F32: v.f = get<float>(); break;
      case GV_F64: v.f = get<double>(); break;
      case GV_STRING: v.s = str(); break;
      default: skip_value(type);  // arrays are skipped; nothing here reads them
    }
    return v;
  }
};

uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // quiet NaN
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const int e = (h >> 10) & 0x1f, m = h & 0x3ff;
  float v;
  if (e == 0) v = std::ldexp((float)m, -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = std::ldexp((float)(m | 0x400), e - 25);
  uint32_t u;
  std::memcpy(&u, &v, 4);
  u |= sign;
  std::memcpy(&v, &u, 4);
  return v;
}

}  // namespace
}  // namespace moe

using namespace moe;

struct moe_gguf {
  void* map = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  std::map<std::string, Value> meta;
  std::vector<TensorInfo> tensors;
  std::map<std::string, size_t> by_name;
  std::vector<std::vector<uint16_t>> owned;  // converted routers
};

extern "C" {

moe_status moe_gguf_open(const char* path, moe_gguf** out) {
  if (!out) return fail(MOE_ERR_INVALID, "moe_gguf_open: null out");
  *out = nullptr;
  if (!path) return fail(MOE_ERR_INVALID, "moe_gguf_open: null path");
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(MOE_ERR_INVALID, std::string("moe_gguf_open: cannot open ") + path);
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 24) {
    close(fd);
    return fail(MOE_ERR_INVALID, std::string("moe_gguf_open: not a GGUF file (too short): ") + path);
  }
  void* map = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (map == MAP_FAILED) return fail(MOE_ERR_INVALID, std::string("moe_gguf_open: mmap failed: ") + path);
  moe_gguf* f = new moe_gguf();
  f->map = map;
  f->size = (size_t)st.st_size;
  auto bad = [&](const std::string& why) {
    munmap(f->map, f->size);
    delete f;
    return fail(MOE_ERR_INVALID, std::string("moe_gguf_open: ") + path + ": " + why);
  };
  Cursor c{static_cast<const uint8_t*>(map), f->size};
  if (std::memcmp(map, "GGUF", 4) != 0) return bad("bad magic (not a GGUF file)");
  c.pos = 4;
  f->version = c.get<uint32_t>();
  if (f->version < 2 || f->version > 3) return bad("unsupported GGUF version " + std::to_string(f->version));
  const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
  if (n_tensors > (1u << 24) || n_kv > (1u << 24)) return bad("implausible tensor or metadata count");
  for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
    std::string key = c.str();
    const uint32_t type = c.get<uint32_t>();
    Value v = c.value(type);
    if (c.ok) f->meta[key] = v;
  }
  if (!c.ok) return bad("truncated or malformed metadata");
  for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
    TensorInfo t;
    t.name = c.str();
    t.n_dims = (int)c.get<uint32_t>();
    if (t.n_dims < 1 || t.n_dims > 4) return bad("tensor " + t.name + ": n_dims out of 1..4");
    for (int d = 0; d < t.n_dims; ++d) {
      const uint64_t v = c.get<uint64_t>();
      if (v == 0 || v > ((uint64_t)1 << 40)) return bad("tensor " + t.name + ": bad dimension");
      t.dims[d] = (int64_t)v;
    }
    t.type = (int)c.get<uint32_t>();
    t.offset = c.get<uint64_t>();
    if (c.ok) {
      f->by_name[t.name] = f->tensors.size();
      f->tensors.push_back(t);
    }
  }
  if (!c.ok) return bad("truncated or malformed tensor table");
  int64_t align = 32;
  auto ai = f->meta.find("general.alignment");
  if (ai != f->meta.end() && ai->second.type <= GV_I64 && ai->second.type != GV_STRING) align = ai->second.i;
  if (align <= 0 || (align & (align - 1))) return bad("general.alignment is not a power of two");
  const size_t data_start = (c.pos + (size_t)align - 1) / (size_t)align * (size_t)align;
  for (auto& t : f->tensors) {
    int64_t blk, bpb;
    ggml_block(t.type, &blk, &bpb);
    if (blk) {
      if (t.dims[0] % blk) return bad("tensor " + t.name + ": first dimension not a multiple of its block");
      int64_t rows = 1;
      for (int d = 1; d < t.n_dims; ++d) rows *= t.dims[d];
      t.nbytes = rows * (t.dims[0] / blk) * bpb;
    }
    const uint64_t at = data_start + t.offset;
    if (at < data_start || at > f->size || (t.nbytes >= 0 && (uint64_t)t.nbytes > f->size - at))
      return bad("tensor " + t.name + ": data past the end of the file");
    t.data = static_cast<const uint8_t*>(map) + at;
  }
  *out = f;
  return MOE_OK;
}

void moe_gguf_close(moe_gguf* f) {
  if (!f) return;
  munmap(f->map, f->size);
  delete f;
}

int moe_gguf_tensor_count(const moe_gguf* f) { return f ? (int)f->tensors.size() : 0; }

const char* moe_gguf_tensor_name(const moe_gguf* f, int i) {
  if (!f || i < 0 || i >= (int)f->tensors.size()) return nullptr;
  return f->tensors[(size_t)i].name.c_str();
}

moe_status moe_gguf_tensor(const moe_gguf* f, const char* name, int* ggml_type, int64_t* dims, int* n_dims,
                           const void** data, int64_t* nbytes) {
  if (!f || !name) return fail(MOE_ERR_INVALID, "moe_gguf_tensor: null argument");
  auto it = f->by_name.find(name);
  if (it == f->by_name.end()) return fail(MOE_ERR_INVALID, std::string("moe_gguf_tensor: no tensor ") + name);
  const TensorInfo& t = f->tensors[it->second];
  if (ggml_type) *ggml_type = t.type;
  if (n_dims) *n_dims = t.n_dims;
  if (dims)
    for (int d = 0; d < 4; ++d) dims[d] = t.dims[d];
  if (data) *data = t.data;
  if (nbytes) *nbytes = t.nbytes;
  return MOE_OK;
}

moe_status moe_gguf_get_int(const moe_gguf* f, const char* key, int64_t* value) {
  if (!f || !key || !value) return fail(MOE_ERR_INVALID, "moe_gguf_get_int: null argument");
  auto it = f->meta.find(key);
  if (it == f->meta.end()) return fail(MOE_ERR_INVALID, std::string("moe_gguf_get_int: no key ") + key);
  const uint32_t t = it->second.type;
  if (t == GV_STRING || t == GV_ARRAY || t == GV_F32 || t == GV_F64)
    return fail(MOE_ERR_INVALID, std::string("moe_gguf_get_int: not an integer: ") + key);
  *value = it->second.i;
  return MOE_OK;
}

size_t moe_gguf_get_str(const moe_gguf* f, const char* key, char* buf, size_t n) {
  if (!f || !key) return 0;
  auto it = f->meta.find(key);
  if (it == f->meta.end() || it->second.type != GV_STRING) return 0;
  const std::string& s = it->second.s;
  if (buf && n) {
    const size_t m = s.size() < n - 1 ? s.size() : n - 1;
    std::memcpy(buf, s.data(), m);
    buf[m] = 0;
  }
  return s.size();
}

moe_status moe_gguf_layer_desc(moe_gguf* f, int layer, moe_layer_desc* d) {
  if (!f || !d || layer < 0) return fail(MOE_ERR_INVALID, "moe_gguf_layer_desc: bad arguments");
  const std::string pre = "blk." + std::to_string(layer) + ".";
  const TensorInfo* proj[3] = {};
  const char* names[3] = {"ffn_gate_exps.weight", "ffn_up_exps.weight", "ffn_down_exps.weight"};
  for (int i = 0; i < 3; ++i) {
    auto it = f->by_name.find(pre + names[i]);
    if (it == f->by_name.end())
      return fail(MOE_ERR_INVALID, "moe_gguf_layer_desc: no tensor " + pre + names[i] + " (not an MoE layer?)");
    proj[i] = &f->tensors[it->second];
    if (proj[i]->n_dims != 3)
      return fail(MOE_ERR_INVALID, "moe_gguf_layer_desc: " + pre + names[i] + " is not a 3-D expert stack");
  }
  const int type = proj[0]->type;
  for (int i = 1; i < 3; ++i)
    if (proj[i]->type != type)
      return fail(MOE_ERR_UNSUPPORTED, "moe_gguf_layer_desc: layer " + std::to_string(layer) +
                                           " mixes weight types across gate/up/down (" + ggml_type_name(type) + ", " +
                                           ggml_type_name(proj[i]->type) + "); one layer runs one type");
  int wdtype;
  switch (type) {
    case GT_Q8_0: wdtype = MOE_DTYPE_Q8_0; break;
    case GT_Q4_K: wdtype = MOE_DTYPE_Q4_K; break;
    case GT_BF16: wdtype = MOE_DTYPE_BF16; break;
    default:
      return fail(MOE_ERR_UNSUPPORTED, "moe_gguf_layer_desc: expert type " + std::to_string(type) +
                                           " is not one this library runs (Q8_0, Q4_K, BF16)");
  }
  // dims[0] = K (fastest), dims[1] = N, dims[2] = E: gate/up [E, I, H], down [E, H, I]
  const int64_t H = proj[0]->dims[0], I = proj[0]->dims[1], E = proj[0]->dims[2];
  if (proj[1]->dims[0] != H || proj[1]->dims[1] != I || proj[1]->dims[2] != E || proj[2]->dims[0] != I ||
      proj[2]->dims[1] != H || proj[2]->dims[2] != E)
    return fail(MOE_ERR_INVALID, "moe_gguf_layer_desc: gate/up/down shapes disagree in layer " + std::to_string(layer));
  if (E > 1024 || H > (1 << 20) || I > (1 << 20))
    return fail(MOE_ERR_INVALID, "moe_gguf_layer_desc: implausible expert shape");
  d->num_experts = (int)E;
  d->hidden = (int)H;
  d->inter = (int)I;
  d->wdtype = wdtype;
  d->gate = proj[0]->data;
  d->up = proj[1]->data;
  d->down = proj[2]->data;
  d->gate_scale = d->up_scale = d->down_scale = nullptr;
  d->weights_on_device = 0;
  // top-k: {architecture}.expert_used_count when the file states it
  char arch[128] = {0};
  if (moe_gguf_get_str(f, "general.architecture", arch, sizeof(arch))) {
    int64_t k = 0;
    auto it = f->meta.find(std::string(arch) + ".expert_used_count");
    if (it != f->meta.end() && it->second.type != GV_STRING && it->second.type != GV_ARRAY) k = it->second.i;
    if (k > 0 && k <= E) d->top_k = (int)k;
  }
  // router: blk.L.ffn_gate_inp.weight [E, H] (dims H, E); bf16 as stored, f32/f16 converted
  d->router_weight = nullptr;
  auto ri = f->by_name.find(pre + "ffn_gate_inp.weight");
  if (ri != f->by_name.end()) {
    const TensorInfo& r = f->tensors[ri->second];
    if (r.n_dims != 2 || r.dims[0] != H || r.dims[1] != E)
      return fail(MOE_ERR_INVALID, "moe_gguf_layer_desc: " + pre + "ffn_gate_inp.weight is not [E, H]");
    const int64_t n = E * H;
    if (r.type == GT_BF16) {
      d->router_weight = reinterpret_cast<const uint16_t*>(r.data);
    } else if (r.type == GT_F32 || r.type == GT_F16) {
      std::vector<uint16_t> bf((size_t)n);
      for (int64_t i = 0; i < n; ++i) {
        float v;
        if (r.type == GT_F32) {
          std::memcpy(&v, r.data + 4 * i, 4);
        } else {
          uint16_t h;
          std::memcpy(&h, r.data + 2 * i, 2);
          v = f16_to_f32(h);
        }
        bf[(size_t)i] = f32_to_bf16_rne(v);
      }
      f->owned.push_back(std::move(bf));
      d->router_weight = f->owned.back().data();
    } else {
      return fail(MOE_ERR_UNSUPPORTED, "moe_gguf_layer_desc: router type " + std::to_string(r.type) +
                                           " is not F32, F16 or BF16");
    }
  }
  return MOE_OK;
}

}  // extern "C"
