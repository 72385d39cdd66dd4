// PBTQW25 v1 layout validation and upload (replaces ModelView::open_authenticated
// of sulewicz/promptboot crates/promptboot-core/src/model.rs:371-629 for the
// decode path), plus the library's host utilities: CUDA error capture, SHA-256
// (FIPS 180-4) and the inference RoPE table.
#include "pb_host.h"
#include "pb_common.cuh"
#include "pb_kernels.cuh"

#include <cmath>

namespace pb {

static thread_local std::string g_last_error;

void set_last_error(const char* text) { g_last_error = text; }

uint32_t record_cuda_error(cudaError_t e, const char* what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return PB_DEVICE;
}

// ----------------------------------------------------------------- SHA-256

namespace {
constexpr uint32_t kK[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4,
    0xab1c5ed5, 0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe,
    0x9bdc06a7, 0xc19bf174, 0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f,
    0x4a7484aa, 0x5cb0a9dc, 0x76f988da, 0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7,
    0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967, 0x27b70a85, 0x2e1b2138, 0x4d2c6dfc,
    0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85, 0xa2bfe8a1, 0xa81a664b,
    0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070, 0x19a4c116,
    0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7,
    0xc67178f2};
inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

void compress(uint32_t h[8], const uint8_t* block) {
  uint32_t w[64];
  for (int i = 0; i < 16; ++i)
    w[i] = (uint32_t)block[4 * i] << 24 | (uint32_t)block[4 * i + 1] << 16 |
           (uint32_t)block[4 * i + 2] << 8 | block[4 * i + 3];
  for (int i = 16; i < 64; ++i) {
    uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
    uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
    w[i] = w[i - 16] + s0 + w[i - 7] + s1;
  }
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], k = h[7];
  for (int i = 0; i < 64; ++i) {
    uint32_t t1 = k + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + kK[i] + w[i];
    uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
    k = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
  }
  h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += k;
}
}  // namespace

void sha256(const uint8_t* data, size_t len, uint8_t out[32]) {
  uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                   0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  size_t full = len / 64;
  for (size_t i = 0; i < full; ++i) compress(h, data + 64 * i);
  uint8_t tail[128] = {};
  size_t rem = len - 64 * full;
  std::memcpy(tail, data + 64 * full, rem);
  tail[rem] = 0x80;
  size_t blocks = rem + 9 > 64 ? 2 : 1;
  uint64_t bits = (uint64_t)len * 8;
  for (int i = 0; i < 8; ++i) tail[blocks * 64 - 1 - i] = (uint8_t)(bits >> (8 * i));
  for (size_t i = 0; i < blocks; ++i) compress(h, tail + 64 * i);
  for (int i = 0; i < 8; ++i)
    for (int j = 0; j < 4; ++j) out[4 * i + j] = (uint8_t)(h[i] >> (24 - 8 * j));
}

bool build_rope_table(std::vector<float>& table) {
  static const uint8_t kPinned[32] = {
      0xcd, 0x75, 0xfc, 0xc6, 0x3f, 0x75, 0x14, 0x05, 0x5d, 0xaf, 0x75, 0x91, 0x75, 0x21, 0xbf, 0xe4,
      0x61, 0x2c, 0xe6, 0x41, 0x74, 0x19, 0xde, 0x5c, 0xe7, 0x7c, 0xa7, 0x66, 0x47, 0x3c, 0x01, 0xc5};
  table.assign((size_t)32768 * 64, 0.0f);
  // volatile keeps the compiler from folding powf with its own (exact) evaluator
  volatile float base = 1000000.0f, expo = -2.0f / 64.0f;
  const float theta_scale = powf(base, expo);
  size_t at = 0;
  for (int position = 0; position < 32768; ++position) {
    float theta = (float)position;
    for (int pair = 0; pair < 32; ++pair) {
      table[at++] = cosf(theta);
      table[at++] = sinf(theta);
      theta = theta * theta_scale;
    }
  }
  uint8_t digest[32];
  sha256(reinterpret_cast<const uint8_t*>(table.data()), table.size() * 4, digest);
  return std::memcmp(digest, kPinned, 32) == 0;
}

}  // namespace pb

// ------------------------------------------------------------- model open

namespace {

inline uint32_t u32_at(const uint8_t* b, size_t o) { uint32_t v; std::memcpy(&v, b + o, 4); return v; }
inline uint16_t u16_at(const uint8_t* b, size_t o) { uint16_t v; std::memcpy(&v, b + o, 2); return v; }
inline uint64_t u64_at(const uint8_t* b, size_t o) { uint64_t v; std::memcpy(&v, b + o, 8); return v; }

// ModelStatus / ErrorDomain / FieldKind numbering of model.rs:10-107
enum : uint32_t {
  M_LENGTH = 1, M_MAGIC = 3, M_VERSION = 4, M_ENDIAN = 5, M_IDENTITY = 6, M_RESERVED = 7,
  M_ARITH = 8, M_ALIGNMENT = 9, M_ORDER = 10, M_OVERLAP = 11, M_PADDING = 12,
  M_SECTION_SCHEMA = 16, M_TENSOR_SCHEMA = 17, M_STATE = 27,
};
enum : uint32_t { DOM_HEADER = 1, DOM_SECTION = 2, DOM_TENSOR = 3 };
enum : uint32_t {
  F_FILE_BYTES = 1, F_BASE_ALIGNMENT = 2, F_DIGEST_BYTE = 3, F_MAGIC_BYTE = 4, F_VERSION = 5,
  F_ENDIAN = 6, F_HEADER_FIELD = 7, F_RESERVED_BYTE = 8, F_SECTION_ID = 9, F_ELEMENT_TYPE = 10,
  F_RANGE_START = 11, F_RANGE_LENGTH = 12, F_GAP_BYTE = 14, F_TENSOR_ID = 15, F_LAYER = 16,
  F_ROLE = 17, F_DTYPE = 18, F_RANK = 19, F_DIMENSION = 20, F_BLOCK_LENGTH = 21, F_OP_ADD = 40,
  F_STATE_FIELD = 39,
};

uint32_t model_error(pb_model_error* err, uint32_t status, uint32_t domain, uint32_t index,
                     uint64_t offset, uint64_t needed, uint64_t available, uint32_t kind,
                     uint32_t sub) {
  if (err) {
    err->status = status; err->domain = domain; err->index = index; err->reserved = 0;
    err->offset = offset; err->needed = needed; err->available = available;
    err->detail = ((uint64_t)kind << 32) | sub;
  }
  return status;
}

const uint64_t kSectionOffsets[7] = {704, 608512, 1981312, 2133248, 3949952, 3952512, 3980480};
const uint64_t kSectionLengths[7] = {607748, 1372758, 151936, 1816644, 2509, 27936, 422782464};
const uint64_t kSectionCounts[7] = {151937, 1372758, 151936, 151387, 2509, 291, 422782464};
const uint32_t kSectionTypes[7] = {1, 2, 2, 3, 2, 4, 2};
const uint8_t kSourceHash[32] = {
    0x76, 0x71, 0xc0, 0xc3, 0x04, 0xe6, 0xce, 0x5a, 0x7f, 0xc5, 0x77, 0xbc, 0xb1, 0x2a, 0xba, 0x01,
    0xe2, 0xc1, 0x55, 0xcc, 0x2e, 0xfd, 0x29, 0xb2, 0x21, 0x3c, 0x95, 0xb1, 0x8e, 0xda, 0xf6, 0xed};

// model.rs:810-833: (layer, role, dtype, rank, dims) of tensor id
struct Expected { uint16_t layer, role; uint32_t dtype, rank, dims[4]; };
Expected expected_tensor(uint32_t id) {
  if (id == 0) return {0xffff, 1, 2, 2, {896, 151936, 1, 1}};
  if (id == 289) return {0xffff, 2, 1, 1, {896, 1, 1, 1}};
  if (id == 290) return {0xffff, 3, 3, 2, {896, 151936, 1, 1}};
  uint16_t layer = (uint16_t)((id - 1) / 12);
  uint32_t slot = (id - 1) % 12;
  uint16_t role = (uint16_t)(10 + slot);
  switch (slot) {
    case 0: case 4: return {layer, role, 1, 1, {896, 1, 1, 1}};
    case 1: return {layer, role, 2, 2, {4864, 896, 1, 1}};
    case 2: case 3: return {layer, role, 2, 2, {896, 4864, 1, 1}};
    case 5: case 10: return {layer, role, 1, 1, {128, 1, 1, 1}};
    case 6: case 11: return {layer, role, 2, 2, {896, 128, 1, 1}};
    case 7: case 9: return {layer, role, 2, 2, {896, 896, 1, 1}};
    default: return {layer, role, 1, 1, {896, 1, 1, 1}};
  }
}

// model.rs:371-620 (header and section directory) and 835-983 (tensor
// directory), in the reference's check order; tokenizer checks are not run.
uint32_t validate_layout(const uint8_t* bytes, uint64_t len, pb_model_error* err, pb_model* m) {
  if (len != pb::kModelBytes)
    return model_error(err, M_LENGTH, DOM_HEADER, 0, 0, pb::kModelBytes, len, F_FILE_BYTES, 0);
  const char magic[8] = {'P', 'B', 'T', 'Q', 'W', '2', '5', '\0'};
  for (int at = 0; at < 8; ++at)
    if (bytes[at] != (uint8_t)magic[at])
      return model_error(err, M_MAGIC, DOM_HEADER, at, at, (uint8_t)magic[at], bytes[at],
                         F_MAGIC_BYTE, at);
  struct E32 { uint32_t off, expected, kind, status; };
  const E32 e32[] = {
      {8, 1, F_VERSION, M_VERSION}, {12, 256, F_HEADER_FIELD, M_IDENTITY},
      {16, 0x01020304, F_ENDIAN, M_ENDIAN}, {20, 7, F_HEADER_FIELD, M_IDENTITY},
      {24, 291, F_HEADER_FIELD, M_IDENTITY}, {28, 151936, F_HEADER_FIELD, M_IDENTITY},
      {32, 151387, F_HEADER_FIELD, M_IDENTITY}, {36, 32768, F_HEADER_FIELD, M_IDENTITY},
      {40, 24, F_HEADER_FIELD, M_IDENTITY}, {44, 896, F_HEADER_FIELD, M_IDENTITY},
      {48, 4864, F_HEADER_FIELD, M_IDENTITY}, {52, 14, F_HEADER_FIELD, M_IDENTITY},
      {56, 2, F_HEADER_FIELD, M_IDENTITY}, {60, 64, F_HEADER_FIELD, M_IDENTITY},
      {64, 151645, F_HEADER_FIELD, M_IDENTITY}, {68, 151643, F_HEADER_FIELD, M_IDENTITY},
      {72, 151643, F_HEADER_FIELD, M_IDENTITY}, {76, 0, F_HEADER_FIELD, M_IDENTITY}};
  for (const E32& e : e32) {
    uint32_t actual = u32_at(bytes, e.off);
    if (actual != e.expected)
      return model_error(err, e.status, DOM_HEADER, e.off, e.off, e.expected, actual, e.kind, 0);
  }
  const uint64_t e64[][2] = {{80, 428730208}, {88, pb::kModelBytes}, {96, 256},
                             {104, 448}, {112, 5947744}, {120, 422782464}};
  for (const auto& e : e64) {
    uint64_t actual = u64_at(bytes, e[0]);
    if (actual != e[1])
      return model_error(err, M_IDENTITY, DOM_HEADER, (uint32_t)e[0], e[0], e[1], actual,
                         F_HEADER_FIELD, 0);
  }
  for (int at = 0; at < 32; ++at)
    if (bytes[128 + at] != kSourceHash[at])
      return model_error(err, M_IDENTITY, DOM_HEADER, 128 + at, 128 + at, kSourceHash[at],
                         bytes[128 + at], F_DIGEST_BYTE, at);
  for (int at = 192; at < 256; ++at)
    if (bytes[at] != 0)
      return model_error(err, M_RESERVED, DOM_HEADER, at, at, 0, bytes[at], F_RESERVED_BYTE, at - 192);
  uint64_t previous_end = 704;
  for (uint32_t ordinal = 0; ordinal < 7; ++ordinal) {
    size_t base = 256 + ordinal * 64;
    uint64_t actual[5] = {u32_at(bytes, base), u32_at(bytes, base + 4), u64_at(bytes, base + 8),
                          u64_at(bytes, base + 16), u64_at(bytes, base + 24)};
    uint64_t expected[5] = {ordinal + 1, kSectionTypes[ordinal], kSectionCounts[ordinal],
                            kSectionOffsets[ordinal], kSectionLengths[ordinal]};
    const uint32_t kinds[5] = {F_SECTION_ID, F_ELEMENT_TYPE, F_RANGE_LENGTH, F_RANGE_START, F_RANGE_LENGTH};
    const uint32_t field_offsets[5] = {0, 4, 8, 16, 24};
    for (int field : {0, 1, 2, 4})
      if (actual[field] != expected[field])
        return model_error(err, M_SECTION_SCHEMA, DOM_SECTION, ordinal, base + field_offsets[field],
                           expected[field], actual[field], kinds[field], field_offsets[field]);
    if (actual[3] & 63)
      return model_error(err, M_ALIGNMENT, DOM_SECTION, ordinal, base + 16, 64, actual[3] & 63,
                         F_RANGE_START, 16);
    if (actual[3] < previous_end)
      return model_error(err, M_OVERLAP, DOM_SECTION, ordinal, base + 16, previous_end, actual[3],
                         F_RANGE_START, 16);
    if (actual[3] != expected[3])
      return model_error(err, M_SECTION_SCHEMA, DOM_SECTION, ordinal, base + 16, expected[3],
                         actual[3], F_RANGE_START, 16);
    for (uint64_t at = previous_end; at < actual[3]; ++at)
      if (bytes[at] != 0)
        return model_error(err, M_PADDING, DOM_SECTION, ordinal, at, 0, bytes[at], F_GAP_BYTE,
                           (uint32_t)(at - previous_end));
    previous_end = actual[3] + actual[4];
  }
  if (previous_end != pb::kModelBytes)
    return model_error(err, M_SECTION_SCHEMA, DOM_SECTION, 6, previous_end, pb::kModelBytes,
                       previous_end, F_RANGE_LENGTH, 0);
  previous_end = kSectionOffsets[6];
  for (uint32_t id = 0; id < 291; ++id) {
    size_t at = pb::kTensorDirectory + (size_t)id * 96;
    Expected x = expected_tensor(id);
    const uint64_t fields[5][2] = {{u32_at(bytes, at), id},
                                   {u16_at(bytes, at + 4), x.layer},
                                   {u16_at(bytes, at + 6), x.role},
                                   {u32_at(bytes, at + 8), x.dtype},
                                   {u32_at(bytes, at + 12), x.rank}};
    const uint32_t kinds[5] = {F_TENSOR_ID, F_LAYER, F_ROLE, F_DTYPE, F_RANK};
    const uint32_t offs[5] = {0, 4, 6, 8, 12};
    for (int f = 0; f < 5; ++f)
      if (fields[f][0] != fields[f][1])
        return model_error(err, M_TENSOR_SCHEMA, DOM_TENSOR, id, at + offs[f], fields[f][1],
                           fields[f][0], kinds[f], 0);
    for (int d = 0; d < 4; ++d) {
      uint32_t dim = u32_at(bytes, at + 16 + 4 * d);
      if (dim != x.dims[d])
        return model_error(err, M_TENSOR_SCHEMA, DOM_TENSOR, id, at + 16 + 4 * d, x.dims[d], dim,
                           F_DIMENSION, d);
    }
    uint64_t elements = (uint64_t)x.dims[0] * x.dims[1] * x.dims[2] * x.dims[3];
    uint64_t length = x.dtype == 1 ? elements * 4 : x.dtype == 2 ? elements / 32 * 18 : elements / 32 * 34;
    uint64_t data_offset = u64_at(bytes, at + 32), data_length = u64_at(bytes, at + 40);
    if (data_length != length)
      return model_error(err, M_TENSOR_SCHEMA, DOM_TENSOR, id, at + 40, length, data_length,
                         F_BLOCK_LENGTH, x.dtype);
    if (data_offset != previous_end)
      return model_error(err, data_offset < previous_end ? M_OVERLAP : M_ORDER, DOM_TENSOR, id,
                         at + 32, previous_end, data_offset, F_RANGE_START, 0);
    if (data_offset & 63)
      return model_error(err, M_ALIGNMENT, DOM_TENSOR, id, at + 32, 64, data_offset & 63,
                         F_RANGE_START, 0);
    for (int r = 80; r < 96; ++r)
      if (bytes[at + r] != 0)
        return model_error(err, M_RESERVED, DOM_TENSOR, id, at + r, 0, bytes[at + r],
                           F_RESERVED_BYTE, r - 80);
    m->offset[id] = data_offset;
    m->length[id] = data_length;
    previous_end = data_offset + data_length;
  }
  if (previous_end != pb::kModelBytes)
    return model_error(err, M_TENSOR_SCHEMA, DOM_TENSOR, 290, previous_end, pb::kModelBytes,
                       previous_end, F_RANGE_LENGTH, 0);
  return 0;
}

}  // namespace

namespace {

// Builds the tensor-core tile image from the uploaded tensors (one repack launch
// per matrix) and waits for it.
cudaError_t build_tc_image(pb_model* m) {
  using pb::launch_tc_repack;
  using pb::tc_image_bytes;
  auto lt = [](int layer, uint32_t role) { return 1u + (uint32_t)layer * 12u + (role - 10u); };
  size_t off = 0;
  for (int l = 0; l < pb::kLayers; ++l) {
    m->tc_qkv[l] = off;
    off += tc_image_bytes(896, 896) + 2 * tc_image_bytes(128, 896);
    m->tc_o[l] = off;
    off += tc_image_bytes(896, 896);
    m->tc_gateup[l] = off;
    off += 2 * tc_image_bytes(4864, 896);
    m->tc_down[l] = off;
    off += tc_image_bytes(896, 4864);
  }
  m->tc_head = off;
  off += tc_image_bytes(pb::kVocab, 896);
  m->tc_bytes = off;
  cudaError_t e = cudaMalloc(&m->tc, off);
  if (e != cudaSuccess) return e;
  for (int l = 0; l < pb::kLayers; ++l) {
    uint8_t* qkv = m->tc + m->tc_qkv[l];
    launch_tc_repack(pb::W_Q4_0, m->tensor(lt(l, 19)), 896, 896, qkv, 0);
    launch_tc_repack(pb::W_Q4_0, m->tensor(lt(l, 16)), 128, 896, qkv + tc_image_bytes(896, 896), 0);
    launch_tc_repack(pb::W_Q4_0, m->tensor(lt(l, 21)), 128, 896,
                     qkv + tc_image_bytes(896, 896) + tc_image_bytes(128, 896), 0);
    launch_tc_repack(pb::W_Q4_0, m->tensor(lt(l, 17)), 896, 896, m->tc + m->tc_o[l], 0);
    uint8_t* gu = m->tc + m->tc_gateup[l];
    launch_tc_repack(pb::W_Q4_0, m->tensor(lt(l, 12)), 4864, 896, gu, 0);
    launch_tc_repack(pb::W_Q4_0, m->tensor(lt(l, 13)), 4864, 896, gu + tc_image_bytes(4864, 896), 0);
    launch_tc_repack(pb::W_Q4_0, m->tensor(lt(l, 11)), 896, 4864, m->tc + m->tc_down[l], 0);
  }
  launch_tc_repack(pb::W_Q8_0, m->tensor(290), pb::kVocab, 896, m->tc + m->tc_head, 0);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  return e;
}

}  // namespace

extern "C" {

uint32_t pb_abi_version(void) { return PB_ABI_VERSION; }

const char* pb_last_error_string(void) { return pb::g_last_error.c_str(); }

uint32_t pb_model_open(const uint8_t* bytes, uint64_t len, uint32_t flags, int device,
                       pb_model** out, pb_model_error* err) {
  if (out) *out = nullptr;
  if (!bytes || !out) return model_error(err, 21, 0, 0, 0, 1, 0, F_STATE_FIELD, 0);
  if (!(flags & PB_MODEL_LAYOUT_ONLY))
    // Authenticated open needs the tokenizer sections (out of this path's scope).
    return model_error(err, M_STATE, DOM_HEADER, 0, 0, PB_MODEL_LAYOUT_ONLY, flags, F_STATE_FIELD, 1);
  pb_model* m = new pb_model();
  uint32_t st = validate_layout(bytes, len, err, m);
  if (st) { delete m; return st; }
  std::vector<float> rope;
  if (!pb::build_rope_table(rope)) {
    delete m;
    return model_error(err, M_STATE, DOM_HEADER, 0, 0, 0, 0, F_DIGEST_BYTE, 2);
  }
  m->device = device;
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaMalloc(&m->data, pb::kTensorDataBytes);
  if (e == cudaSuccess) e = cudaMemcpy(m->data, bytes + pb::kTensorSection, pb::kTensorDataBytes,
                                       cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&m->rope, rope.size() * 4);
  if (e == cudaSuccess) e = cudaMemcpy(m->rope, rope.data(), rope.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = build_tc_image(m);
  if (e != cudaSuccess) {
    pb::record_cuda_error(e, "pb_model_open");
    if (m->data) cudaFree(m->data);
    if (m->rope) cudaFree(m->rope);
    if (m->tc) cudaFree(m->tc);
    delete m;
    return model_error(err, PB_DEVICE, 0, 0, 0, 0, (uint64_t)e, F_STATE_FIELD, 3);
  }
  *out = m;
  if (err) std::memset(err, 0, sizeof *err);
  return 0;
}

void pb_model_close(pb_model* model) {
  if (!model) return;
  cudaSetDevice(model->device);
  if (model->data) cudaFree(model->data);
  if (model->rope) cudaFree(model->rope);
  if (model->tc) cudaFree(model->tc);
  if (model->tc_embed) cudaFree(model->tc_embed);
  if (model->op_scratch) cudaFree(model->op_scratch);
  if (model->op_status) cudaFree(model->op_status);
  delete model;
}

const void* pb_model_tensor_device(const pb_model* model, uint32_t id) {
  if (!model || id >= 291) return nullptr;
  return model->tensor(id);
}

uint32_t pb_rope_table(float* table_host) {
  std::vector<float> t;
  bool ok = pb::build_rope_table(t);
  if (table_host) std::memcpy(table_host, t.data(), t.size() * 4);
  return ok ? 0 : PB_MODEL;
}

}  // extern "C"
