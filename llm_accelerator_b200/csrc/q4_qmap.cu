// QMAP v1 blob consumption: walk the reference's per-layer runtime packets in
// a host copy of the PL-DDR arena and bind every model tensor they describe.
//
// Format: Source/QMAP_FORMAT.md (256-byte header :134-184, 128-byte tensor
// descriptor :186-214, role / dtype / flag enums :216-263, per-packet slot
// tables :546-1814).  Layout of the deployed full28 image: packet bases per
// layer from FPGA_Project/software/qmap_one_token_runtime/
// qmap_model_config_generated.h (qot_layer_qmap_bases_t order,
// qmap_one_token_runtime.h:31-42), persistent weight offsets from
// Qwen3-0.6B-Base/python_each_module/53_export_embedding_full28_final_chain.py:21-75.
//
// Tensors are found by meaning, not by slot number (QMAP_FORMAT.md:278-280):
// Q4 weights by role + matrix id (aux0) with the scale their scale_tensor_id
// names, gammas / LUTs by role, dtype and length, the RoPE planes by role.
// Everything is host code; q4gpu_model_load_qmap then uploads through
// q4gpu_model_set_tensor.
#include <cstring>
#include <vector>

#include "q4gpu_internal.h"

namespace {

constexpr uint32_t kMagic = 0x50414D51u;  // "QMAP", little-endian
enum : uint32_t {
  kRoleWeight = 2, kRoleScale = 3, kRoleMetadata = 6, kRoleRope = 8, kRoleParam = 9,
};
enum : uint32_t {
  kDtU32 = 5, kDtI32 = 6, kDtPackedQ4 = 16, kDtU16Q2_14 = 17, kDtI16Q8_7 = 22, kDtI16Q1_15 = 23, kDtU32Q0_20 = 24,
  kDtU16Q0_16 = 25,
};
enum : uint32_t { kMatQ = 1, kMatK, kMatV, kMatO, kMatGate, kMatUp, kMatDown, kMatEmbed };
// qot_layer_qmap_bases_t field order
enum { kQkv = 0, kInputNorm, kFrontend, kScoreValue, kOProj, kPostNorm, kGateUp, kSiluMul, kDown, kResidual };
constexpr int kLayerBaseCount = 10;
constexpr uint32_t kScoreScaleQ0_31 = 189812531u;  // round(128^-1/2 * 2^31)

struct Arena {
  const uint8_t* p;
  uint64_t base, bytes;
  // arena offset of [addr, addr + n), false when it leaves the arena
  bool span(uint64_t addr, uint64_t n, uint64_t* off) const {
    if (addr < base) return false;
    const uint64_t o = addr - base;
    if (o > bytes || n > bytes - o) return false;
    *off = o;
    return true;
  }
};

struct Packet {
  uint64_t addr = 0;
  q4gpu_qmap_header h{};
  std::vector<q4gpu_qmap_descriptor> d;
};

int bad(const char* what, uint64_t addr) {
  return q4gpu_fail(Q4GPU_ERR_ARG, "QMAP: %s (packet 0x%llx)", what, (unsigned long long)addr);
}

int read_packet(const Arena& a, uint64_t addr, Packet& pk) {
  static_assert(sizeof(q4gpu_qmap_descriptor) == 128, "descriptor is 128 bytes");
  uint64_t off;
  if (!a.span(addr, 256, &off)) return bad("header outside the arena", addr);
  q4gpu_qmap_header& h = pk.h;
  std::memcpy(&h, a.p + off, sizeof(h));
  if (h.magic != kMagic) return bad("bad magic", addr);
  if (h.version != 1u) return bad("unsupported version", addr);
  if (h.header_bytes != 256u || h.descriptor_bytes != 128u) return bad("bad header/descriptor size", addr);
  if (h.descriptor_count > h.descriptor_capacity || h.descriptor_capacity > 4096u)
    return bad("descriptor count above capacity", addr);
  if (h.image_base_addr != addr) return bad("image_base_addr differs from the packet address", addr);
  if (h.descriptor_table_addr < addr + 256u) return bad("descriptor table overlaps the header", addr);
  uint64_t toff;
  if (!a.span(h.descriptor_table_addr, (uint64_t)h.descriptor_count * 128u, &toff))
    return bad("descriptor table outside the arena", addr);
  pk.addr = addr;
  pk.d.resize(h.descriptor_count);
  if (h.descriptor_count) std::memcpy(pk.d.data(), a.p + toff, (size_t)h.descriptor_count * 128u);
  return Q4GPU_OK;
}

const q4gpu_qmap_descriptor* by_id(const Packet& pk, uint32_t id) {
  for (const auto& d : pk.d)
    if (d.tensor_id == id) return &d;
  return nullptr;
}

// Q4 weight of matrix `mat` (rows x cols, packed low-even, row stride cols / 2)
// and its U16 Q2.14 scale (rows x cols / 64, row stride cols / 32).
int bind_weight(const Arena& a, const Packet& pk, uint32_t mat, int layer, int32_t which, int rows, int cols,
                q4gpu_qmap_tensor* t) {
  const q4gpu_qmap_descriptor* w = nullptr;
  for (const auto& d : pk.d)
    if (d.role == kRoleWeight && d.aux[0] == mat) {
      w = &d;
      break;
    }
  if (!w) return bad("Q4 weight descriptor missing", pk.addr);
  if (w->dtype != kDtPackedQ4 || w->rank != 2 || w->element_bits != 4)
    return bad("Q4 weight is not PACKED_Q4_S4 rank 2", pk.addr);
  if (layer >= 0 && w->aux[1] != (uint32_t)layer) return bad("Q4 weight belongs to another layer", pk.addr);
  if ((rows > 0 && w->dims[0] != (uint32_t)rows) || w->dims[1] != (uint32_t)cols ||
      w->strides_bytes[0] != (uint64_t)cols / 2)
    return bad("Q4 weight shape or row stride", pk.addr);
  const q4gpu_qmap_descriptor* s = by_id(pk, w->scale_tensor_id);
  if (!s || s->role != kRoleScale || s->dtype != kDtU16Q2_14) return bad("Q4 scale descriptor", pk.addr);
  if (s->dims[0] != w->dims[0] || s->dims[1] != (uint32_t)(cols / 64) || s->strides_bytes[0] != (uint64_t)cols / 32 ||
      (s->strides_bytes[1] != 2u && s->strides_bytes[1] != 0u))
    return bad("Q4 scale shape or stride", pk.addr);
  const uint64_t wb = (uint64_t)w->dims[0] * (cols / 2), sb = (uint64_t)w->dims[0] * (cols / 32);
  if (w->nbytes < wb || s->nbytes < sb) return bad("Q4 payload shorter than its shape", pk.addr);
  q4gpu_qmap_tensor r{};
  r.layer = layer;
  r.which = which;
  r.rows = (int32_t)w->dims[0];
  r.cols = cols;
  r.data_bytes = wb;
  r.scale_bytes = sb;
  if (!a.span(w->base_addr, wb, &r.data_offset) || !a.span(s->base_addr, sb, &r.scale_offset))
    return bad("Q4 payload outside the arena", pk.addr);
  r.elem_kind = Q4GPU_QMAP_PACKED_Q4;
  *t = r;
  return Q4GPU_OK;
}

// The n-th PARAMETER descriptor of dtype `dt` and length `count` (slot order).
int bind_param(const Arena& a, const Packet& pk, uint32_t dt, int count, int nth, int layer, int32_t which,
               q4gpu_qmap_tensor* t) {
  int seen = 0;
  for (const auto& d : pk.d) {
    if (d.role != kRoleParam || d.dtype != dt || d.dims[0] != (uint32_t)count) continue;
    if (seen++ != nth) continue;
    const uint64_t stride = d.strides_bytes[0];
    const bool narrow = dt == kDtI16Q8_7 || dt == kDtU16Q0_16;
    if (!(stride == 4u || (narrow && stride == 2u))) return bad("parameter element stride", pk.addr);
    const uint64_t nb = stride * (uint64_t)count;
    if (d.nbytes < nb) return bad("parameter payload shorter than its shape", pk.addr);
    q4gpu_qmap_tensor r{};
    r.layer = layer;
    r.which = which;
    r.rows = count;
    r.data_bytes = nb;
    r.elem_stride = (int32_t)stride;
    r.elem_kind = dt == kDtI16Q8_7 ? Q4GPU_QMAP_S16 : (dt == kDtU16Q0_16 ? Q4GPU_QMAP_U16 : Q4GPU_QMAP_U32);
    if (!a.span(d.base_addr, nb, &r.data_offset)) return bad("parameter payload outside the arena", pk.addr);
    *t = r;
    return Q4GPU_OK;
  }
  return bad("parameter descriptor missing", pk.addr);
}

// RoPE plane from the front-end packet: the persistent runtime table
// [positions, 128] (rank 2, row stride 512 B) that every layer points at.
int bind_rope(const Arena& a, const Packet& pk, int nth, int32_t which, q4gpu_qmap_tensor* t) {
  int seen = 0;
  for (const auto& d : pk.d) {
    if (d.role != kRoleRope) continue;
    if (seen++ != nth) continue;
    if (d.dtype != kDtI16Q1_15) return bad("RoPE plane is not I16_Q1_15", pk.addr);
    if (d.rank != 2 || d.dims[1] != 128u || d.strides_bytes[0] != 512u || d.strides_bytes[1] != 4u)
      return bad("RoPE descriptor is not the rank-2 runtime table", pk.addr);
    const uint64_t nb = (uint64_t)d.dims[0] * 512u;
    q4gpu_qmap_tensor r{};
    r.layer = -1;
    r.which = which;
    r.rows = (int32_t)d.dims[0];
    r.cols = 128;
    r.data_bytes = nb;
    r.elem_stride = 4;
    r.elem_kind = Q4GPU_QMAP_S16;
    if (!a.span(d.base_addr, nb, &r.data_offset)) return bad("RoPE table outside the arena", pk.addr);
    *t = r;
    return Q4GPU_OK;
  }
  return bad("RoPE descriptor missing", pk.addr);
}

bool same_bytes(const Arena& a, const q4gpu_qmap_tensor& x, const q4gpu_qmap_tensor& y) {
  return x.data_bytes == y.data_bytes && x.elem_stride == y.elem_stride &&
         std::memcmp(a.p + x.data_offset, a.p + y.data_offset, (size_t)x.data_bytes) == 0;
}

// Element i of a bound vector as an int32 (16-bit values sign- or zero-
// extended from their slot); false if a 32-bit slot does not hold a valid
// extension of its 16-bit value.
bool vec_elem(const Arena& a, const q4gpu_qmap_tensor& t, int64_t i, int32_t* out) {
  const uint8_t* p = a.p + t.data_offset + (uint64_t)i * t.elem_stride;
  if (t.elem_stride == 2) {
    uint16_t v;
    std::memcpy(&v, p, 2);
    *out = t.elem_kind == Q4GPU_QMAP_S16 ? (int32_t)(int16_t)v : (int32_t)v;
    return true;
  }
  uint32_t w;
  std::memcpy(&w, p, 4);
  if (t.elem_kind == Q4GPU_QMAP_S16) {
    *out = (int32_t)w;
    return *out >= -32768 && *out <= 32767;
  }
  if (t.elem_kind == Q4GPU_QMAP_U16) {  // UQ0.16 stored in a word: 1.0 = 65536 is representable
    *out = (int32_t)w;
    return w <= 65536u;
  }
  *out = (int32_t)w;
  return w <= 0x7FFFFFFFu;
}

}  // namespace

extern "C" {

int q4gpu_qmap_read_packet(const uint8_t* arena, uint64_t arena_base, uint64_t arena_bytes, uint64_t packet_addr,
                           q4gpu_qmap_header* header, q4gpu_qmap_descriptor* desc, int32_t desc_cap) {
  if (!arena || !header || (desc_cap > 0 && !desc)) return q4gpu_fail(Q4GPU_ERR_ARG, "null QMAP argument");
  const Arena a{arena, arena_base, arena_bytes};
  Packet pk;
  const int rc = read_packet(a, packet_addr, pk);
  if (rc != Q4GPU_OK) return rc;
  *header = pk.h;
  const int n = (int)pk.d.size() < desc_cap ? (int)pk.d.size() : desc_cap;
  if (n > 0) std::memcpy(desc, pk.d.data(), (size_t)n * sizeof(q4gpu_qmap_descriptor));
  return (int)pk.d.size();
}

int q4gpu_qmap_bind(const uint8_t* arena, uint64_t arena_bytes, const q4gpu_qmap_layout* layout,
                    q4gpu_qmap_tensor* out, int32_t cap, int32_t* n_out) {
  if (!arena || !layout || !n_out || (cap > 0 && !out) || !layout->layer_bases || layout->n_layers < 1)
    return q4gpu_fail(Q4GPU_ERR_ARG, "null or empty QMAP layout");
  const Arena a{arena, layout->arena_base, arena_bytes};
  std::vector<q4gpu_qmap_tensor> ts;
  q4gpu_qmap_tensor t;
  int rc;
  auto push = [&](const q4gpu_qmap_tensor& x) { ts.push_back(x); };
  q4gpu_qmap_tensor exp0{}, sig0{}, rope_cos{}, rope_sin{};
  for (int l = 0; l < layout->n_layers; ++l) {
    const uint64_t* b = layout->layer_bases + (size_t)l * kLayerBaseCount;
    if (!b[kQkv] || !b[kInputNorm] || !b[kFrontend] || !b[kScoreValue] || !b[kOProj] || !b[kPostNorm] ||
        !b[kGateUp] || !b[kSiluMul] || !b[kDown] || !b[kResidual])
      return q4gpu_fail(Q4GPU_ERR_ARG, "QMAP: layer %d base table has a zero entry", l);
    Packet qkv, in_norm, front, sv, o, post, gu, silu, down, resid;
    if ((rc = read_packet(a, b[kQkv], qkv)) || (rc = read_packet(a, b[kInputNorm], in_norm)) ||
        (rc = read_packet(a, b[kFrontend], front)) || (rc = read_packet(a, b[kScoreValue], sv)) ||
        (rc = read_packet(a, b[kOProj], o)) || (rc = read_packet(a, b[kPostNorm], post)) ||
        (rc = read_packet(a, b[kGateUp], gu)) || (rc = read_packet(a, b[kSiluMul], silu)) ||
        (rc = read_packet(a, b[kDown], down)) || (rc = read_packet(a, b[kResidual], resid)))
      return rc;
    if ((rc = bind_weight(a, qkv, kMatQ, l, Q4GPU_T_Q, 2048, 1024, &t))) return rc;
    push(t);
    if ((rc = bind_weight(a, qkv, kMatK, l, Q4GPU_T_K, 1024, 1024, &t))) return rc;
    push(t);
    if ((rc = bind_weight(a, qkv, kMatV, l, Q4GPU_T_V, 1024, 1024, &t))) return rc;
    push(t);
    if ((rc = bind_weight(a, o, kMatO, l, Q4GPU_T_O, 1024, 2048, &t))) return rc;
    push(t);
    if ((rc = bind_weight(a, gu, kMatGate, l, Q4GPU_T_GATE, 3072, 1024, &t))) return rc;
    push(t);
    if ((rc = bind_weight(a, gu, kMatUp, l, Q4GPU_T_UP, 3072, 1024, &t))) return rc;
    push(t);
    if ((rc = bind_weight(a, down, kMatDown, l, Q4GPU_T_DOWN, 1024, 3072, &t))) return rc;
    push(t);
    if ((rc = bind_param(a, in_norm, kDtI16Q8_7, 1024, 0, l, Q4GPU_T_INPUT_GAMMA, &t))) return rc;
    push(t);
    if ((rc = bind_param(a, post, kDtI16Q8_7, 1024, 0, l, Q4GPU_T_POST_GAMMA, &t))) return rc;
    push(t);
    // front-end slots 4 and 5: q_norm then k_norm gamma
    if ((rc = bind_param(a, front, kDtI16Q8_7, 128, 0, l, Q4GPU_T_Q_GAMMA, &t))) return rc;
    push(t);
    if ((rc = bind_param(a, front, kDtI16Q8_7, 128, 1, l, Q4GPU_T_K_GAMMA, &t))) return rc;
    push(t);
    // one softmax exp LUT and one sigmoid LUT serve every layer
    q4gpu_qmap_tensor e, s;
    if ((rc = bind_param(a, sv, kDtU32Q0_20, 257, 0, -1, Q4GPU_T_EXP_LUT, &e))) return rc;
    if ((rc = bind_param(a, silu, kDtU16Q0_16, 1025, 0, -1, Q4GPU_T_SIGMOID_LUT, &s))) return rc;
    if (l == 0) {
      exp0 = e;
      sig0 = s;
      q4gpu_qmap_tensor c{}, sn{};
      if ((rc = bind_rope(a, front, 0, Q4GPU_T_ROPE_COS, &c)) || (rc = bind_rope(a, front, 1, Q4GPU_T_ROPE_SIN, &sn)))
        return rc;
      if (layout->rope_cos_base && (c.data_offset != layout->rope_cos_base - layout->arena_base))
        return bad("RoPE cos plane differs from the layout's runtime table", b[kFrontend]);
      if (layout->rope_sin_base && (sn.data_offset != layout->rope_sin_base - layout->arena_base))
        return bad("RoPE sin plane differs from the layout's runtime table", b[kFrontend]);
      rope_cos = c;
      rope_sin = sn;
      push(c);
      push(sn);
    } else {
      if (!same_bytes(a, e, exp0) || !same_bytes(a, s, sig0))
        return q4gpu_fail(Q4GPU_ERR_ARG, "QMAP: layer %d LUTs differ from layer 0's", l);
      q4gpu_qmap_tensor c{}, sn{};
      if ((rc = bind_rope(a, front, 0, Q4GPU_T_ROPE_COS, &c)) || (rc = bind_rope(a, front, 1, Q4GPU_T_ROPE_SIN, &sn)))
        return rc;
      if (c.data_offset != rope_cos.data_offset || sn.data_offset != rope_sin.data_offset ||
          c.rows != rope_cos.rows)
        return q4gpu_fail(Q4GPU_ERR_ARG, "QMAP: layer %d points at another RoPE table", l);
    }
    for (const auto& d : sv.d)
      if (d.role == kRoleMetadata && d.aux[0] != kScoreScaleQ0_31)
        return bad("attention score scale differs from round(2^31 / sqrt(128))", b[kScoreValue]);
  }
  ts.push_back(exp0);
  ts.push_back(sig0);
  Packet tail;
  if ((rc = read_packet(a, layout->final_tail_qmap_base, tail))) return rc;
  if ((rc = bind_weight(a, tail, kMatEmbed, -1, Q4GPU_T_EMBED, 0, 1024, &t))) return rc;
  t.layer = -1;
  if ((layout->embed_weight_base && t.data_offset != layout->embed_weight_base - layout->arena_base) ||
      (layout->embed_scale_base && t.scale_offset != layout->embed_scale_base - layout->arena_base))
    return bad("LM-head descriptors differ from the layout's tied embedding", layout->final_tail_qmap_base);
  push(t);
  if ((rc = bind_param(a, tail, kDtI16Q8_7, 1024, 0, -1, Q4GPU_T_FINAL_GAMMA, &t))) return rc;
  push(t);
  *n_out = (int32_t)ts.size();
  if ((int)ts.size() > cap) return cap > 0 ? q4gpu_fail(Q4GPU_ERR_WORKSPACE, "QMAP: %d tensors, room for %d",
                                                        (int)ts.size(), cap)
                                           : Q4GPU_OK;
  std::memcpy(out, ts.data(), ts.size() * sizeof(q4gpu_qmap_tensor));
  return Q4GPU_OK;
}

int q4gpu_qmap_vector(const uint8_t* arena, const q4gpu_qmap_tensor* t, int32_t* out, int64_t count) {
  if (!arena || !t || !out) return q4gpu_fail(Q4GPU_ERR_ARG, "null QMAP argument");
  if (t->elem_kind == Q4GPU_QMAP_PACKED_Q4 || t->elem_stride <= 0) return q4gpu_fail(Q4GPU_ERR_ARG, "not a vector");
  const int64_t n = (int64_t)(t->data_bytes / (uint64_t)t->elem_stride);
  if (count != n) return q4gpu_fail(Q4GPU_ERR_SHAPE, "QMAP vector holds %lld values", (long long)n);
  const Arena a{arena, 0, ~0ull};
  for (int64_t i = 0; i < n; ++i)
    if (!vec_elem(a, *t, i, out + i))
      return q4gpu_fail(Q4GPU_ERR_ARG, "QMAP vector element %lld is not a valid %s value", (long long)i,
                        t->elem_kind == Q4GPU_QMAP_S16 ? "sign-extended 16-bit" : "unsigned");
  return Q4GPU_OK;
}

int q4gpu_model_load_qmap(q4gpu_model* m, const uint8_t* arena, uint64_t arena_bytes,
                          const q4gpu_qmap_layout* layout) {
  if (!m || !arena || !layout) return q4gpu_fail(Q4GPU_ERR_ARG, "null model/arena/layout");
  int n = 0;
  int rc = q4gpu_qmap_bind(arena, arena_bytes, layout, nullptr, 0, &n);
  if (rc != Q4GPU_OK) return rc;
  std::vector<q4gpu_qmap_tensor> ts(n);
  if ((rc = q4gpu_qmap_bind(arena, arena_bytes, layout, ts.data(), n, &n))) return rc;
  q4gpu_model_config cfg{};
  q4gpu_model_get_config(m, &cfg);
  if (layout->n_layers != cfg.n_layers)
    return q4gpu_fail(Q4GPU_ERR_SHAPE, "QMAP image has %d layers, the model %d", layout->n_layers, cfg.n_layers);
  std::vector<int32_t> v;
  for (const auto& t : ts) {
    if (t.elem_kind == Q4GPU_QMAP_PACKED_Q4) {
      if (t.which == Q4GPU_T_EMBED && t.rows != cfg.vocab)
        return q4gpu_fail(Q4GPU_ERR_SHAPE, "QMAP LM head has %d rows, the model's vocab is %d", t.rows, cfg.vocab);
      rc = q4gpu_model_set_tensor(m, t.layer < 0 ? 0 : t.layer, t.which, arena + t.data_offset, (size_t)t.data_bytes,
                                  reinterpret_cast<const uint16_t*>(arena + t.scale_offset), (size_t)t.scale_bytes);
      if (rc) return rc;
      continue;
    }
    const int64_t count = (int64_t)(t.data_bytes / (uint64_t)t.elem_stride);
    if (t.which == Q4GPU_T_ROPE_COS || t.which == Q4GPU_T_ROPE_SIN) {
      // the image's positions replace the model's first rows; positions
      // past the image (extended context) keep the model's own table
      v.assign((size_t)cfg.max_context * 128, 0);
      if ((rc = q4gpu_model_get_tensor(m, 0, t.which, v.data(), v.size() * 4, nullptr, 0))) return rc;
      std::vector<int32_t> img((size_t)count);
      if ((rc = q4gpu_qmap_vector(arena, &t, img.data(), count))) return rc;
      const int rows = t.rows < cfg.max_context ? t.rows : cfg.max_context;
      std::memcpy(v.data(), img.data(), (size_t)rows * 128 * 4);
    } else {
      v.assign((size_t)count, 0);
      if ((rc = q4gpu_qmap_vector(arena, &t, v.data(), count))) return rc;
    }
    if ((rc = q4gpu_model_set_tensor(m, t.layer < 0 ? 0 : t.layer, t.which, v.data(), v.size() * 4, nullptr, 0)))
      return rc;
  }
  return Q4GPU_OK;
}

}  // extern "C"
