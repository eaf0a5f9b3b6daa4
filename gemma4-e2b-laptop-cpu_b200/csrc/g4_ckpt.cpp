// Checkpoint reader: the reference's weight loading (gemma4_engine.cpp:1211-1231) in library form.
// The reference mmaps <ckpt>/model.safetensors and finds each tensor through an index file that
// tools/make_index.py writes from the safetensors header (one line per tensor: name, dtype,
// absolute offset, byte count, comma-separated shape).  g4_checkpoint_open reads that index, or,
// without one, the header itself (8-byte little-endian length, then a JSON object name ->
// {"dtype", "shape", "data_offsets" relative to the end of the header}), and maps the file.  Every
// tensor's extent is checked against the file and its byte count against dtype x shape.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <fstream>
#include <sstream>

#include "g4_api.h"
#include "g4_ckpt.h"
#include "g4_model.cuh"

using g4::CkTensor;
using g4::set_error;

namespace {

size_t dtype_size(const std::string& d) {
  if (d == "BF16" || d == "F16" || d == "I16" || d == "U16") return 2;
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  if (d == "U8" || d == "I8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
  return 0;
}

// A minimal JSON reader for the safetensors header: objects, arrays, strings, numbers, literals.
struct Json {
  const char* p;
  const char* end;
  bool ok = true;
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool eat(char c) {
    ws();
    if (p < end && *p == c) { ++p; return true; }
    return false;
  }
  bool str(std::string& out) {
    ws();
    if (p >= end || *p != '"') return ok = false;
    ++p;
    out.clear();
    while (p < end && *p != '"') {
      if (*p == '\\') {
        if (++p >= end) return ok = false;
        switch (*p) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {  // kept as the escape text: tensor names are ASCII
            if (end - p < 5) return ok = false;
            out += "\\u";
            out.append(p + 1, 4);
            p += 4;
            break;
          }
          default: out += *p;
        }
        ++p;
      } else {
        out += *p++;
      }
    }
    if (p >= end) return ok = false;
    ++p;
    return true;
  }
  bool integer(long long& v) {
    ws();
    const char* s = p;
    if (p < end && *p == '-') ++p;
    if (p >= end || *p < '0' || *p > '9') return ok = false;
    while (p < end && *p >= '0' && *p <= '9') ++p;
    v = std::strtoll(std::string(s, p).c_str(), nullptr, 10);
    return true;
  }
  int depth = 0;
  bool skip() {  // any value (nesting bounded: a header is a flat object of small objects)
    ws();
    if (p >= end || depth > 64) return ok = false;
    if (*p == '"') { std::string s; return str(s); }
    if (*p == '{' || *p == '[') {
      const char close = *p == '{' ? '}' : ']';
      const bool obj = *p == '{';
      ++p;
      if (eat(close)) return true;
      ++depth;
      do {
        if (obj) {
          std::string k;
          if (!str(k) || !eat(':')) return ok = false;
        }
        if (!skip()) return false;
      } while (eat(','));
      --depth;
      if (!eat(close)) ok = false;
      return ok;
    }
    while (p < end && *p != ',' && *p != '}' && *p != ']' && *p != ' ' && *p != '\n') ++p;
    return true;
  }
  bool int_array(std::vector<long long>& out) {
    out.clear();
    if (!eat('[')) return ok = false;
    if (eat(']')) return true;
    do {
      long long v;
      if (!integer(v)) return false;
      out.push_back(v);
    } while (eat(','));
    if (!eat(']')) ok = false;
    return ok;
  }
};

int parse_header(g4_checkpoint& ck) {
  if (ck.size < 8) return set_error(G4_ERR_INVALID, "checkpoint %s: shorter than a safetensors header", ck.path.c_str());
  uint64_t n = 0;
  std::memcpy(&n, ck.base, 8);
  if (n > ck.size - 8) return set_error(G4_ERR_INVALID, "checkpoint %s: header length %llu past the end", ck.path.c_str(), (unsigned long long)n);
  const size_t data0 = 8 + (size_t)n;
  Json j{reinterpret_cast<const char*>(ck.base) + 8, reinterpret_cast<const char*>(ck.base) + data0};
  if (!j.eat('{')) return set_error(G4_ERR_INVALID, "checkpoint %s: header is not a JSON object", ck.path.c_str());
  if (!j.eat('}')) {
    do {
      std::string name;
      if (!j.str(name) || !j.eat(':')) break;
      if (name == "__metadata__") {
        if (!j.skip()) break;
        continue;
      }
      CkTensor t;
      std::vector<long long> offs;
      if (!j.eat('{')) { j.ok = false; break; }
      if (!j.eat('}')) {
        do {
          std::string key;
          if (!j.str(key) || !j.eat(':')) { j.ok = false; break; }
          if (key == "dtype") j.str(t.dtype);
          else if (key == "shape") j.int_array(t.shape);
          else if (key == "data_offsets") j.int_array(offs);
          else j.skip();
          if (!j.ok) break;
        } while (j.eat(','));
        if (!j.ok || !j.eat('}')) { j.ok = false; break; }
      }
      if (offs.size() != 2 || offs[0] < 0 || offs[1] < offs[0])
        return set_error(G4_ERR_INVALID, "checkpoint %s: tensor %s has no valid data_offsets", ck.path.c_str(), name.c_str());
      t.off = data0 + (size_t)offs[0];
      t.nbytes = (size_t)(offs[1] - offs[0]);
      ck.t[name] = t;
    } while (j.eat(','));
    if (j.ok && !j.eat('}')) j.ok = false;
  }
  if (!j.ok) return set_error(G4_ERR_INVALID, "checkpoint %s: malformed safetensors header", ck.path.c_str());
  return G4_OK;
}

int parse_index(g4_checkpoint& ck, const char* index) {
  std::ifstream f(index);
  if (!f) return set_error(G4_ERR_INVALID, "checkpoint index %s: cannot open", index);
  std::string line;
  int ln = 0;
  while (std::getline(f, line)) {
    ++ln;
    if (line.empty()) continue;
    std::stringstream ss(line);
    std::string name, dtype, off, nb, shape;
    std::getline(ss, name, '\t');
    std::getline(ss, dtype, '\t');
    std::getline(ss, off, '\t');
    std::getline(ss, nb, '\t');
    std::getline(ss, shape, '\t');
    CkTensor t;
    t.dtype = dtype;
    char* e1 = nullptr;
    char* e2 = nullptr;
    const unsigned long long o = std::strtoull(off.c_str(), &e1, 10), b = std::strtoull(nb.c_str(), &e2, 10);
    if (name.empty() || off.empty() || nb.empty() || *e1 || *e2)
      return set_error(G4_ERR_INVALID, "checkpoint index %s: line %d is not name, dtype, offset, bytes, shape", index, ln);
    t.off = (size_t)o;
    t.nbytes = (size_t)b;
    std::stringstream s2(shape);
    std::string x;
    while (std::getline(s2, x, ',')) {
      char* e3 = nullptr;
      const long long v = std::strtoll(x.c_str(), &e3, 10);
      if (x.empty() || *e3 || v < 0) return set_error(G4_ERR_INVALID, "checkpoint index %s: line %d has a bad shape", index, ln);
      t.shape.push_back(v);
    }
    ck.t[name] = t;
  }
  return G4_OK;
}

int check_tensors(const g4_checkpoint& ck) {
  for (auto& kv : ck.t) {
    const CkTensor& t = kv.second;
    const size_t es = dtype_size(t.dtype);
    if (es == 0) return set_error(G4_ERR_UNSUPPORTED, "checkpoint: tensor %s has dtype %s", kv.first.c_str(), t.dtype.c_str());
    size_t count = 1;
    for (long long s : t.shape) count *= (size_t)s;
    if (count * es != t.nbytes)
      return set_error(G4_ERR_INVALID, "checkpoint: tensor %s holds %zu bytes, its dtype and shape need %zu", kv.first.c_str(),
                       t.nbytes, count * es);
    if (t.off > ck.size || t.nbytes > ck.size - t.off)
      return set_error(G4_ERR_INVALID, "checkpoint: tensor %s lies past the end of %s", kv.first.c_str(), ck.path.c_str());
  }
  return G4_OK;
}

const CkTensor* need(const g4_checkpoint* ck, const std::string& name, const char* dtype, std::vector<long long> shape,
                     int* rc) {
  const CkTensor* t = ck->find(name);
  if (!t) {
    *rc = set_error(G4_ERR_INVALID, "checkpoint: tensor %s missing", name.c_str());
    return nullptr;
  }
  if (t->dtype != dtype || t->shape != shape) {
    std::string want, got;
    for (long long s : shape) want += (want.empty() ? "" : ",") + std::to_string(s);
    for (long long s : t->shape) got += (got.empty() ? "" : ",") + std::to_string(s);
    *rc = set_error(G4_ERR_INVALID, "checkpoint: tensor %s is %s [%s], expected %s [%s]", name.c_str(), t->dtype.c_str(),
                    got.c_str(), dtype, want.c_str());
    return nullptr;
  }
  *rc = G4_OK;
  return t;
}

// The int4 matrix of `base` (weight_packed as I32 [N][K/8], the compressed-tensors form the
// reference reads, or U8 [N][K/2]; weight_scale BF16 [N][K/32]).
const CkTensor* need_packed(const g4_checkpoint* ck, const std::string& base, long long N, long long K, int* rc) {
  const std::string name = base + ".weight_packed";
  const CkTensor* t = ck->find(name);
  if (t && t->dtype == "U8") return need(ck, name, "U8", {N, K / 2}, rc);
  return need(ck, name, "I32", {N, K / 8}, rc);
}

}  // namespace

std::string g4::ck_layer(int l, const char* suffix) { return "layers." + std::to_string(l) + "." + suffix; }

int g4::ck_load_lin(const g4_checkpoint* ck, const std::vector<std::pair<std::string, int>>& parts, int K, uint8_t* w_dev,
                    uint16_t* s_dev, cudaStream_t st) {
  size_t ro = 0, so = 0;
  for (auto& p : parts) {
    int rc = G4_OK;
    const CkTensor* w = need_packed(ck, p.first, p.second, K, &rc);
    if (!w) return rc;
    const CkTensor* s = need(ck, p.first + ".weight_scale", "BF16", {p.second, K / 32}, &rc);
    if (!s) return rc;
    if (cudaMemcpyAsync(w_dev + ro, ck->base + w->off, w->nbytes, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(reinterpret_cast<uint8_t*>(s_dev) + so, ck->base + s->off, s->nbytes, cudaMemcpyHostToDevice, st) !=
            cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
      return set_error(G4_ERR_CUDA, "checkpoint: copy of %s failed", p.first.c_str());
    ro += w->nbytes;
    so += s->nbytes;
  }
  return G4_OK;
}

int g4::ck_load_vec(const g4_checkpoint* ck, const std::string& name, int n, float* dev, cudaStream_t st) {
  int rc = G4_OK;
  const CkTensor* t = need(ck, name, "BF16", {n}, &rc);
  if (!t) return rc;
  std::vector<float> v((size_t)n);
  for (int i = 0; i < n; ++i) {
    uint16_t b;
    std::memcpy(&b, ck->base + t->off + 2 * (size_t)i, 2);
    const uint32_t u = (uint32_t)b << 16;
    std::memcpy(&v[(size_t)i], &u, 4);
  }
  if (cudaMemcpyAsync(dev, v.data(), sizeof(float) * (size_t)n, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)  // before v goes out of scope
    return set_error(G4_ERR_CUDA, "checkpoint: copy of %s failed", name.c_str());
  return G4_OK;
}

int g4::ck_load_bf16(const g4_checkpoint* ck, const std::string& name, long long rows, long long cols, uint16_t* dev,
                     cudaStream_t st) {
  int rc = G4_OK;
  const CkTensor* t = need(ck, name, "BF16", {rows, cols}, &rc);
  if (!t) return rc;
  if (cudaMemcpyAsync(dev, ck->base + t->off, t->nbytes, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return set_error(G4_ERR_CUDA, "checkpoint: copy of %s failed", name.c_str());
  return G4_OK;
}

int g4::ck_load_scalar(const g4_checkpoint* ck, const std::string& name, float* out) {
  const CkTensor* t = ck->find(name);
  if (!t) {
    *out = 1.0f;
    return G4_OK;
  }
  if (t->dtype != "BF16" || t->nbytes != 2)
    return set_error(G4_ERR_INVALID, "checkpoint: tensor %s is not one bf16 value", name.c_str());
  uint16_t b;
  std::memcpy(&b, ck->base + t->off, 2);
  const uint32_t u = (uint32_t)b << 16;
  std::memcpy(out, &u, 4);
  return G4_OK;
}

extern "C" int g4_checkpoint_open(const char* path, const char* index, g4_checkpoint** out) {
  if (!path || !out) return set_error(G4_ERR_INVALID, "g4_checkpoint_open: null pointer");
  *out = nullptr;
  std::string file = path;
  struct stat sb;
  if (stat(path, &sb) == 0 && S_ISDIR(sb.st_mode)) file += "/model.safetensors";  // the reference's <ckpt> directory
  g4_checkpoint* ck = new g4_checkpoint();
  ck->path = file;
  ck->fd = open(file.c_str(), O_RDONLY);
  if (ck->fd < 0 || fstat(ck->fd, &sb) != 0) {
    delete ck;
    return set_error(G4_ERR_INVALID, "g4_checkpoint_open: cannot open %s", file.c_str());
  }
  ck->size = (size_t)sb.st_size;
  if (ck->size > 0) {
    void* m = mmap(nullptr, ck->size, PROT_READ, MAP_PRIVATE, ck->fd, 0);
    if (m == MAP_FAILED) {
      g4_checkpoint_close(ck);
      return set_error(G4_ERR_INVALID, "g4_checkpoint_open: cannot map %s", file.c_str());
    }
    ck->base = static_cast<const uint8_t*>(m);
  }
  int rc = index ? parse_index(*ck, index) : parse_header(*ck);
  if (rc == G4_OK) rc = check_tensors(*ck);
  if (rc != G4_OK) {
    g4_checkpoint_close(ck);
    return rc;
  }
  *out = ck;
  return G4_OK;
}

extern "C" void g4_checkpoint_close(g4_checkpoint* ck) {
  if (!ck) return;
  if (ck->base) munmap(const_cast<uint8_t*>(ck->base), ck->size);
  if (ck->fd >= 0) close(ck->fd);
  delete ck;
}

extern "C" int g4_checkpoint_tensor(const g4_checkpoint* ck, const char* name, char* dtype, int dtype_cap,
                                    long long* shape, int shape_cap, int* ndim, long long* nbytes) {
  if (!ck || !name) return set_error(G4_ERR_INVALID, "g4_checkpoint_tensor: null pointer");
  const CkTensor* t = ck->find(name);
  if (!t) return set_error(G4_ERR_INVALID, "g4_checkpoint_tensor: no tensor %s", name);
  if (dtype && dtype_cap > 0) {
    std::strncpy(dtype, t->dtype.c_str(), (size_t)dtype_cap - 1);
    dtype[dtype_cap - 1] = 0;
  }
  if (ndim) *ndim = (int)t->shape.size();
  if (shape)
    for (int i = 0; i < (int)t->shape.size() && i < shape_cap; ++i) shape[i] = t->shape[(size_t)i];
  if (nbytes) *nbytes = (long long)t->nbytes;
  return G4_OK;
}

extern "C" int g4_checkpoint_count(const g4_checkpoint* ck) { return ck ? (int)ck->t.size() : 0; }

// The model sizes of the checkpoint, with every tensor the engine reads checked (name, dtype,
// shape), and the parts of the real E2B model this build does not run reported by name.
extern "C" int g4_checkpoint_config(const g4_checkpoint* ck, g4_engine_config* cfg) {
  if (!ck || !cfg) return set_error(G4_ERR_INVALID, "g4_checkpoint_config: null pointer");
  int rc = G4_OK;
  const CkTensor* E = ck->find("embed_tokens.weight");
  if (!E || E->dtype != "BF16" || E->shape.size() != 2)
    return set_error(G4_ERR_INVALID, "checkpoint: embed_tokens.weight missing or not a bf16 matrix");
  const long long V = E->shape[0], H = E->shape[1];
  int NL = 0;
  while (ck->find(g4::ck_layer(NL, "input_layernorm.weight"))) ++NL;
  if (NL == 0) return set_error(G4_ERR_INVALID, "checkpoint: no layers.0.input_layernorm.weight");
  const CkTensor* g0 = ck->find(g4::ck_layer(0, "mlp.gate_proj.weight_scale"));
  if (!g0 || g0->shape.size() != 2) return set_error(G4_ERR_INVALID, "checkpoint: layers.0.mlp.gate_proj missing");
  const long long I = g0->shape[0];
  const CkTensor* kn0 = ck->find(g4::ck_layer(0, "self_attn.k_norm.weight"));
  if (!kn0 || kn0->shape.size() != 1) return set_error(G4_ERR_INVALID, "checkpoint: layers.0.self_attn.k_norm.weight missing");
  constexpr long long HD = 256, NQ = 8;
  // KV sharing (owner_of, gemma4_engine.cpp:1251): the layers from the first one without k/v
  // projections on read their owner's cache; every one of them must lack them and have an owner
  int OWN = 0;
  while (OWN < NL && ck->find(g4::ck_layer(OWN, "self_attn.k_proj.weight_scale"))) ++OWN;
  if (OWN == NL) OWN = 0;
  g4::ModelDims dd;
  dd.NL = NL;
  dd.OWN = OWN;
  for (int l = 0; l < NL; ++l) {
    if (!dd.owns(l) && (ck->find(g4::ck_layer(l, "self_attn.k_proj.weight_scale")) ||
                        ck->find(g4::ck_layer(l, "self_attn.v_proj.weight_scale"))))
      return set_error(G4_ERR_UNSUPPORTED, "checkpoint: layer %d has k/v projections after the KV-shared layer %d (the "
                       "shared layers must be the last ones)", l, OWN);
    if (dd.owner_of(l) < 0)
      return set_error(G4_ERR_UNSUPPORTED, "checkpoint: KV-shared layer %d has no %s layer to read its cache from", l,
                       dd.global_layer(l) ? "global" : "sliding");
  }
  // MLP widths: one for the owners (layer 0's), one for the KV-shared layers (the E2B model
  // doubles it there)
  long long IS = I;
  if (OWN > 0) {
    const CkTensor* gs = ck->find(g4::ck_layer(OWN, "mlp.gate_proj.weight_scale"));
    if (gs && gs->shape.size() == 2) IS = gs->shape[0];
  }
  for (int l = 0; l < NL; ++l) {
    const CkTensor* kn = ck->find(g4::ck_layer(l, "self_attn.k_norm.weight"));
    if (kn && kn->shape.size() == 1 && kn->shape[0] != HD)
      return set_error(G4_ERR_UNSUPPORTED, "checkpoint: layer %d has head_dim %lld (this build runs head_dim 256)", l, kn->shape[0]);
    const long long Il = dd.owns(l) ? I : IS;
    const CkTensor* gl = ck->find(g4::ck_layer(l, "mlp.gate_proj.weight_scale"));
    if (gl && gl->shape.size() == 2 && gl->shape[0] != Il)
      return set_error(G4_ERR_UNSUPPORTED, "checkpoint: layer %d has MLP width %lld, expected %lld (one width for the owner "
                       "layers and one for the KV-shared layers in this build)", l, gl->shape[0], Il);
    const std::string p = "layers." + std::to_string(l) + ".";
    const std::pair<const char*, std::pair<long long, long long>> lins[] = {
        {"self_attn.q_proj", {NQ * HD, H}}, {"self_attn.k_proj", {HD, H}}, {"self_attn.v_proj", {HD, H}},
        {"self_attn.o_proj", {H, NQ * HD}}, {"mlp.gate_proj", {Il, H}},     {"mlp.up_proj", {Il, H}},
        {"mlp.down_proj", {H, Il}}};
    for (auto& li : lins) {
      if (!dd.owns(l) && (!std::strcmp(li.first, "self_attn.k_proj") || !std::strcmp(li.first, "self_attn.v_proj"))) continue;
      const std::string b = p + li.first;
      if (!need_packed(ck, b, li.second.first, li.second.second, &rc)) return rc;
      if (!need(ck, b + ".weight_scale", "BF16", {li.second.first, li.second.second / 32}, &rc)) return rc;
    }
    const std::pair<const char*, long long> vecs[] = {{"input_layernorm.weight", H},  {"post_attention_layernorm.weight", H},
                                                      {"pre_feedforward_layernorm.weight", H}, {"post_feedforward_layernorm.weight", H},
                                                      {"self_attn.q_norm.weight", HD}, {"self_attn.k_norm.weight", HD}};
    for (auto& v : vecs) {
      if (!dd.owns(l) && !std::strcmp(v.first, "self_attn.k_norm.weight")) continue;
      if (!need(ck, p + v.first, "BF16", {v.second}, &rc)) return rc;
    }
    float s;
    if ((rc = g4::ck_load_scalar(ck, p + "layer_scalar", &s)) != G4_OK) return rc;
  }
  if (!need(ck, "norm.weight", "BF16", {H}, &rc)) return rc;
  // per-layer embeddings (PLE, :1230-1231, 1226-1229): 256 inputs per layer
  const bool ple = ck->find("embed_tokens_per_layer.weight") || ck->find("per_layer_model_projection.weight_scale");
  if (ple) {
    const long long NP = 256LL * NL;
    if (!need(ck, "embed_tokens_per_layer.weight", "BF16", {V, NP}, &rc)) return rc;
    if (!need_packed(ck, "per_layer_model_projection", NP, H, &rc)) return rc;
    if (!need(ck, "per_layer_model_projection.weight_scale", "BF16", {NP, H / 32}, &rc)) return rc;
    if (!need(ck, "per_layer_projection_norm.weight", "BF16", {256}, &rc)) return rc;
    for (int l = 0; l < NL; ++l) {
      const std::string p = "layers." + std::to_string(l) + ".";
      if (!need_packed(ck, p + "per_layer_input_gate", 256, H, &rc)) return rc;
      if (!need(ck, p + "per_layer_input_gate.weight_scale", "BF16", {256, H / 32}, &rc)) return rc;
      if (!need_packed(ck, p + "per_layer_projection", H, 256, &rc)) return rc;
      if (!need(ck, p + "per_layer_projection.weight_scale", "BF16", {H, 256 / 32}, &rc)) return rc;
      if (!need(ck, p + "post_per_layer_input_norm.weight", "BF16", {H}, &rc)) return rc;
    }
  }
  cfg->ple = ple ? 1 : 0;
  cfg->hidden = (int)H;
  cfg->n_layers = NL;
  cfg->kv_owners = OWN;
  cfg->mlp_shared = IS != I ? (int)IS : 0;
  cfg->mlp = (int)I;
  cfg->vocab = (int)V;
  return G4_OK;
}
