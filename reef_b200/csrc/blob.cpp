// blob.cpp -- loading reef's packed GPT-Neo model ("REEF" blob v1).
//
// The layout is reef's firmware format (coral/include/reef_kernels/
// model_blob.hpp:18-66, read in place by coral/firmware/gpt_neo.cc:61-97;
// written by coral/host/pack_model.hpp:88-160):
// little-endian, a fixed header, every array at a 16-byte-aligned byte offset,
// linear weights stored transposed ([in][out]) with float row scales for
// W8A8, and a table of per-layer records.  The structs below restate that
// layout field for field (the format must be alike to be read at all).
//
// Reading the header needs no GPU.  Loading a layer copies its arrays into a
// caller-provided device arena and repacks each [in][out] int8 weight into
// the K-major [out][kpad(in)] layout the tcgen05 GEMM reads (pack_weight_i8,
// through a staging area in the same arena), then fills a GPT-Neo block
// descriptor with the pointers.  Loading a model puts the token and position
// tables and ln_f first, then one such layer arena per layer, and fills a
// model descriptor (the firmware's GptNeo constructor reads the blob in
// place instead).  A float blob's layers keep their [in][out] weights, which
// the exact float linear reads as they are.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "ops.h"
#include "reef_b200.h"

namespace reef {
namespace {

constexpr uint32_t kMagic = 0x46454552u;  // "REEF"
constexpr uint32_t kVersion = 1;
constexpr uint32_t kPrecisionF32 = 0, kPrecisionW8A8 = 1;

struct Linear {  // BlobLinear
  uint32_t weight, scales;
};

struct Layer {  // BlobLayer
  uint32_t ln_1_weight, ln_1_bias;
  Linear query, key, value, output;
  uint32_t output_bias;
  uint32_t ln_2_weight, ln_2_bias;
  Linear fc;
  uint32_t fc_bias;
  Linear proj;
  uint32_t proj_bias;
  uint32_t is_local;
};

struct Header {  // BlobHeader
  uint32_t magic, version, precision;
  uint32_t vocab_size, max_positions, hidden_size, num_layers, num_heads, inner_size,
      window_size;
  float layer_norm_eps;
  uint32_t wte, wpe, ln_f_weight, ln_f_bias, layers, total_bytes;
};

static_assert(sizeof(Layer) == 80 && sizeof(Header) == 68, "reef's blob records");

// [off, off + bytes) inside the blob's `total` bytes, off 16-byte aligned
bool span_ok(uint64_t off, uint64_t bytes, uint64_t total) {
  return off % 16 == 0 && off <= total && bytes <= total - off;
}

int read_header(const void* blob, size_t bytes, Header* h) {
  if (blob == nullptr || bytes < sizeof(Header)) return kErrInvalid;
  std::memcpy(h, blob, sizeof(Header));
  if (h->magic != kMagic || h->version != kVersion) return kErrInvalid;
  if (h->precision != kPrecisionF32 && h->precision != kPrecisionW8A8) return kErrInvalid;
  const uint64_t total = h->total_bytes;
  if (total < sizeof(Header) || total > bytes) return kErrInvalid;
  if (h->vocab_size == 0 || h->max_positions == 0 || h->hidden_size == 0 ||
      h->num_layers == 0 || h->num_heads == 0 || h->inner_size == 0 ||
      h->hidden_size % h->num_heads != 0)
    return kErrInvalid;
  const uint64_t d = h->hidden_size;
  if (!span_ok(h->wte, uint64_t{h->vocab_size} * d * 4, total) ||
      !span_ok(h->wpe, uint64_t{h->max_positions} * d * 4, total) ||
      !span_ok(h->ln_f_weight, d * 4, total) || !span_ok(h->ln_f_bias, d * 4, total) ||
      !span_ok(h->layers, uint64_t{h->num_layers} * sizeof(Layer), total))
    return kErrInvalid;
  return kOk;
}

size_t al256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

struct Arena {  // byte offsets of one layer's arrays in the device arena
  size_t wq, wk, wv, wo, wfc, wproj, stage;
  size_t sq, sk, sv, so, bo, ln1g, ln1b, ln2g, ln2b, sproj, bproj, sfc, bfc;
  size_t end;
};

Arena arena_layout(size_t d, size_t f) {
  const size_t kd = kpad(d);
  const size_t kf = kpad(f);
  Arena a{};
  size_t at = 0;
  auto take = [&](size_t bytes) {
    const size_t o = at;
    at += al256(bytes);
    return o;
  };
  a.wq = take(d * kd);
  a.wk = take(d * kd);
  a.wv = take(d * kd);
  a.wo = take(d * kd);
  a.wfc = take(f * kd);
  a.wproj = take(d * kf);
  a.stage = take(d * f > d * d ? d * f : d * d);  // one [in][out] weight before packing
  for (size_t* p : {&a.sq, &a.sk, &a.sv, &a.so, &a.bo, &a.ln1g, &a.ln1b, &a.ln2g, &a.ln2b,
                    &a.sproj, &a.bproj})
    *p = take(d * 4);
  a.sfc = take(f * 4);
  a.bfc = take(f * 4);
  a.end = at;
  return a;
}

struct ArenaF32 {  // byte offsets of one float layer's arrays (weights kept [in][out])
  size_t wq, wk, wv, wo, wfc, wproj;
  size_t bo, ln1g, ln1b, ln2g, ln2b, bproj, bfc;
  size_t end;
};

ArenaF32 arena_layout_f32(size_t d, size_t f) {
  ArenaF32 a{};
  size_t at = 0;
  auto take = [&](size_t bytes) {
    const size_t o = at;
    at += al256(bytes);
    return o;
  };
  a.wq = take(d * d * 4);
  a.wk = take(d * d * 4);
  a.wv = take(d * d * 4);
  a.wo = take(d * d * 4);
  a.wfc = take(d * f * 4);
  a.wproj = take(f * d * 4);
  for (size_t* p : {&a.bo, &a.ln1g, &a.ln1b, &a.ln2g, &a.ln2b, &a.bproj}) *p = take(d * 4);
  a.bfc = take(f * 4);
  a.end = at;
  return a;
}

struct ModelArena {  // byte offsets of the model-level arrays, then the layers
  size_t wte, wpe, ln_f_g, ln_f_b, layers, layer_bytes, end;
};

ModelArena model_layout(size_t vocab, size_t positions, size_t d, size_t layers, size_t f,
                        bool w8a8) {
  ModelArena m{};
  size_t at = 0;
  auto take = [&](size_t bytes) {
    const size_t o = at;
    at += al256(bytes);
    return o;
  };
  m.wte = take(vocab * d * 4);
  m.wpe = take(positions * d * 4);
  m.ln_f_g = take(d * 4);
  m.ln_f_b = take(d * 4);
  m.layer_bytes = w8a8 ? arena_layout(d, f).end : arena_layout_f32(d, f).end;
  m.layers = at;
  m.end = at + layers * m.layer_bytes;
  return m;
}

// Copies float layer `layer` of a validated float blob into `dst` (device)
// and fills the block.  Every span is checked before anything is copied.
int load_layer_f32(const Header& h, const uint8_t* src, size_t layer, uint8_t* dst,
                   reef_b200_gptneo_block_f32* block, cudaStream_t st) {
  Layer L;
  std::memcpy(&L, src + h.layers + layer * sizeof(Layer), sizeof(Layer));
  const uint64_t total = h.total_bytes, d = h.hidden_size, f = h.inner_size;
  const ArenaF32 a = arena_layout_f32(d, f);
  const struct {
    uint32_t off;
    uint64_t bytes;
    size_t to;
  } arrays[] = {{L.ln_1_weight, d * 4, a.ln1g},   {L.ln_1_bias, d * 4, a.ln1b},
                {L.query.weight, d * d * 4, a.wq}, {L.key.weight, d * d * 4, a.wk},
                {L.value.weight, d * d * 4, a.wv}, {L.output.weight, d * d * 4, a.wo},
                {L.output_bias, d * 4, a.bo},      {L.ln_2_weight, d * 4, a.ln2g},
                {L.ln_2_bias, d * 4, a.ln2b},      {L.fc.weight, d * f * 4, a.wfc},
                {L.fc_bias, f * 4, a.bfc},         {L.proj.weight, f * d * 4, a.wproj},
                {L.proj_bias, d * 4, a.bproj}};
  for (const auto& r : arrays)
    if (!span_ok(r.off, r.bytes, total)) return REEF_B200_ERR_INVALID;
  for (const auto& r : arrays)
    if (cudaMemcpyAsync(dst + r.to, src + r.off, r.bytes, cudaMemcpyHostToDevice, st) !=
        cudaSuccess)
      return REEF_B200_ERR_CUDA;
  auto f32 = [&](size_t o) { return reinterpret_cast<const float*>(dst + o); };
  block->seq = 0;
  block->hidden = d;
  block->heads = h.num_heads;
  block->head_dim = d / h.num_heads;
  block->ffn = f;
  block->window = L.is_local ? h.window_size : 0;
  block->eps = h.layer_norm_eps;
  block->ln1_g = f32(a.ln1g);
  block->ln1_b = f32(a.ln1b);
  block->wq = f32(a.wq);
  block->wk = f32(a.wk);
  block->wv = f32(a.wv);
  block->wo = f32(a.wo);
  block->bo = f32(a.bo);
  block->ln2_g = f32(a.ln2g);
  block->ln2_b = f32(a.ln2b);
  block->wfc = f32(a.wfc);
  block->bfc = f32(a.bfc);
  block->wproj = f32(a.wproj);
  block->bproj = f32(a.bproj);
  return REEF_B200_OK;
}

bool model_size_ok(size_t vocab, size_t positions, size_t d, size_t layers, size_t f) {
  return d > 0 && f > 0 && d <= (1u << 20) && f <= (1u << 22) && vocab <= (1u << 24) &&
         positions <= (1u << 24) && layers <= 4096;
}

}  // namespace
}  // namespace reef

using namespace reef;

extern "C" {

int reef_b200_blob_read_info(const void* blob, size_t bytes, reef_b200_blob_info* info) {
  if (info == nullptr) return REEF_B200_ERR_INVALID;
  Header h;
  if (int rc = read_header(blob, bytes, &h)) return rc;
  info->precision = h.precision;
  info->vocab = h.vocab_size;
  info->max_positions = h.max_positions;
  info->hidden = h.hidden_size;
  info->layers = h.num_layers;
  info->heads = h.num_heads;
  info->inner = h.inner_size;
  info->window = h.window_size;
  info->eps = h.layer_norm_eps;
  info->wte = h.wte;
  info->wpe = h.wpe;
  info->ln_f_weight = h.ln_f_weight;
  info->ln_f_bias = h.ln_f_bias;
  return REEF_B200_OK;
}

size_t reef_b200_blob_layer_bytes(const reef_b200_blob_info* info) {
  if (info == nullptr || info->hidden == 0 || info->inner == 0 || info->hidden > (1u << 20) ||
      info->inner > (1u << 22))
    return 0;
  return arena_layout(info->hidden, info->inner).end;
}

int reef_b200_blob_load_layer(const void* blob, size_t bytes, size_t layer, void* arena,
                              size_t arena_bytes, reef_b200_gptneo_block* block,
                              reef_b200_stream_t stream) {
  if (arena == nullptr || block == nullptr) return REEF_B200_ERR_INVALID;
  Header h;
  if (int rc = read_header(blob, bytes, &h)) return rc;
  // the kernels here run W8A8 blocks; a float blob is reef's other mode
  if (h.precision != kPrecisionW8A8) return REEF_B200_ERR_UNSUPPORTED;
  if (layer >= h.num_layers) return REEF_B200_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(arena) % 256 != 0) return REEF_B200_ERR_ALIGNMENT;
  const size_t d = h.hidden_size, f = h.inner_size;
  if (d > (1u << 20) || f > (1u << 22)) return REEF_B200_ERR_TOO_LARGE;
  const Arena a = arena_layout(d, f);
  if (arena_bytes < a.end) return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  Layer L;
  std::memcpy(&L, static_cast<const uint8_t*>(blob) + h.layers + layer * sizeof(Layer),
              sizeof(Layer));
  const uint64_t total = h.total_bytes;
  // every array of the layer inside the blob before anything is copied
  {
    const uint64_t D = d, F = f;
    const struct {
      uint32_t off;
      uint64_t bytes;
    } spans[] = {{L.ln_1_weight, D * 4},  {L.ln_1_bias, D * 4},     {L.query.weight, D * D},
                 {L.query.scales, D * 4}, {L.key.weight, D * D},    {L.key.scales, D * 4},
                 {L.value.weight, D * D}, {L.value.scales, D * 4},  {L.output.weight, D * D},
                 {L.output.scales, D * 4}, {L.output_bias, D * 4},  {L.ln_2_weight, D * 4},
                 {L.ln_2_bias, D * 4},    {L.fc.weight, D * F},     {L.fc.scales, F * 4},
                 {L.fc_bias, F * 4},      {L.proj.weight, F * D},   {L.proj.scales, D * 4},
                 {L.proj_bias, D * 4}};
    for (const auto& sp : spans)
      if (!span_ok(sp.off, sp.bytes, total)) return REEF_B200_ERR_INVALID;
  }
  const auto* src = static_cast<const uint8_t*>(blob);
  auto* dst = static_cast<uint8_t*>(arena);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // float arrays straight into place
  auto floats = [&](uint32_t off, size_t n, size_t to) -> int {
    if (!span_ok(off, n * 4, total)) return REEF_B200_ERR_INVALID;
    return cudaMemcpyAsync(dst + to, src + off, n * 4, cudaMemcpyHostToDevice, st) == cudaSuccess
               ? REEF_B200_OK
               : REEF_B200_ERR_CUDA;
  };
  // an int8 [in][out] weight through the staging area, repacked [out][kpad(in)]
  auto weight = [&](uint32_t off, size_t in, size_t out, size_t to) -> int {
    if (!span_ok(off, in * out, total)) return REEF_B200_ERR_INVALID;
    if (cudaMemcpyAsync(dst + a.stage, src + off, in * out, cudaMemcpyHostToDevice, st) !=
        cudaSuccess)
      return REEF_B200_ERR_CUDA;
    return pack_weight_i8(static_cast<long long>(in), static_cast<long long>(out),
                          reinterpret_cast<const int8_t*>(dst + a.stage),
                          reinterpret_cast<int8_t*>(dst + to), static_cast<long long>(kpad(in)),
                          st);
  };
  int rc = REEF_B200_OK;
  auto run = [&](int r) {
    if (rc == REEF_B200_OK) rc = r;
  };
  run(floats(L.ln_1_weight, d, a.ln1g));
  run(floats(L.ln_1_bias, d, a.ln1b));
  run(weight(L.query.weight, d, d, a.wq));
  run(floats(L.query.scales, d, a.sq));
  run(weight(L.key.weight, d, d, a.wk));
  run(floats(L.key.scales, d, a.sk));
  run(weight(L.value.weight, d, d, a.wv));
  run(floats(L.value.scales, d, a.sv));
  run(weight(L.output.weight, d, d, a.wo));
  run(floats(L.output.scales, d, a.so));
  run(floats(L.output_bias, d, a.bo));
  run(floats(L.ln_2_weight, d, a.ln2g));
  run(floats(L.ln_2_bias, d, a.ln2b));
  run(weight(L.fc.weight, d, f, a.wfc));
  run(floats(L.fc.scales, f, a.sfc));
  run(floats(L.fc_bias, f, a.bfc));
  run(weight(L.proj.weight, f, d, a.wproj));
  run(floats(L.proj.scales, d, a.sproj));
  run(floats(L.proj_bias, d, a.bproj));
  if (rc != REEF_B200_OK) return rc;
  auto f32 = [&](size_t o) { return reinterpret_cast<const float*>(dst + o); };
  auto i8 = [&](size_t o) { return reinterpret_cast<const int8_t*>(dst + o); };
  block->hidden = d;
  block->heads = h.num_heads;
  block->head_dim = d / h.num_heads;
  block->ffn = f;
  block->window = L.is_local ? h.window_size : 0;  // odd layers are local (weights.hpp:62)
  block->eps = h.layer_norm_eps;
  block->ln1_g = f32(a.ln1g);
  block->ln1_b = f32(a.ln1b);
  block->wq = i8(a.wq);
  block->sq = f32(a.sq);
  block->wk = i8(a.wk);
  block->sk = f32(a.sk);
  block->wv = i8(a.wv);
  block->sv = f32(a.sv);
  block->wo = i8(a.wo);
  block->so = f32(a.so);
  block->bo = f32(a.bo);
  block->ln2_g = f32(a.ln2g);
  block->ln2_b = f32(a.ln2b);
  block->wfc = i8(a.wfc);
  block->sfc = f32(a.sfc);
  block->bfc = f32(a.bfc);
  block->wproj = i8(a.wproj);
  block->sproj = f32(a.sproj);
  block->bproj = f32(a.bproj);
  return REEF_B200_OK;
}

size_t reef_b200_blob_model_bytes(const reef_b200_blob_info* info) {
  if (info == nullptr ||
      !model_size_ok(info->vocab, info->max_positions, info->hidden, info->layers, info->inner))
    return 0;
  return model_layout(info->vocab, info->max_positions, info->hidden, info->layers, info->inner,
                      info->precision == kPrecisionW8A8)
      .end;
}

int reef_b200_blob_load_model(const void* blob, size_t bytes, void* arena, size_t arena_bytes,
                              reef_b200_gptneo_model* model, reef_b200_gptneo_block* blocks,
                              reef_b200_gptneo_block_f32* blocks_f32,
                              reef_b200_stream_t stream) {
  if (arena == nullptr || model == nullptr) return REEF_B200_ERR_INVALID;
  Header h;
  if (int rc = read_header(blob, bytes, &h)) return rc;
  const bool w8a8 = h.precision == kPrecisionW8A8;
  if ((w8a8 && blocks == nullptr) || (!w8a8 && blocks_f32 == nullptr))
    return REEF_B200_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(arena) % 256 != 0) return REEF_B200_ERR_ALIGNMENT;
  const size_t v = h.vocab_size, n = h.max_positions, d = h.hidden_size, f = h.inner_size;
  if (!model_size_ok(v, n, d, h.num_layers, f)) return REEF_B200_ERR_TOO_LARGE;
  const ModelArena ma = model_layout(v, n, d, h.num_layers, f, w8a8);
  if (arena_bytes < ma.end) return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  const auto* src = static_cast<const uint8_t*>(blob);
  auto* dst = static_cast<uint8_t*>(arena);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the tables and ln_f (read_header checked their spans)
  const struct {
    uint32_t off;
    size_t bytes, to;
  } arrays[] = {{h.wte, v * d * 4, ma.wte},
                {h.wpe, n * d * 4, ma.wpe},
                {h.ln_f_weight, d * 4, ma.ln_f_g},
                {h.ln_f_bias, d * 4, ma.ln_f_b}};
  for (const auto& a : arrays)
    if (cudaMemcpyAsync(dst + a.to, src + a.off, a.bytes, cudaMemcpyHostToDevice, st) !=
        cudaSuccess)
      return REEF_B200_ERR_CUDA;
  for (size_t l = 0; l < h.num_layers; ++l) {
    uint8_t* at = dst + ma.layers + l * ma.layer_bytes;
    const int rc = w8a8 ? reef_b200_blob_load_layer(blob, bytes, l, at, ma.layer_bytes,
                                                    &blocks[l], stream)
                        : load_layer_f32(h, src, l, at, &blocks_f32[l], st);
    if (rc != REEF_B200_OK) return rc;
  }
  auto f32 = [&](size_t o) { return reinterpret_cast<const float*>(dst + o); };
  model->vocab = v;
  model->max_positions = n;
  model->hidden = d;
  model->layers = h.num_layers;
  model->eps = h.layer_norm_eps;
  model->wte = f32(ma.wte);
  model->wpe = f32(ma.wpe);
  model->ln_f_g = f32(ma.ln_f_g);
  model->ln_f_b = f32(ma.ln_f_b);
  model->blocks = w8a8 ? blocks : nullptr;
  model->blocks_f32 = w8a8 ? nullptr : blocks_f32;
  return REEF_B200_OK;
}

}  // extern "C"
