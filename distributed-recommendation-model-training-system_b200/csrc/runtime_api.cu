// runtime_api.cu -- eps_runtime_api_v1: the reference's framework-facing C ABI
// (include/eps/runtime_c.h, adapters/entropy/runtime_c.cpp) served by the B200
// store, so that a consumer which loads a runtime by that symbol (the
// TensorFlow ops, adapters/entropy/tensorflow_ops.cc:38-52) can load this
// library unchanged.
//
// One runtime = one local shard (an EpsB200Store on the configured GPU) behind
// the adapter's batch lifecycle (adapters/entropy/table_adapter.cpp):
//   handles numbered from 0, live / completed maps, the live-batch limit,
//   read-only batches (auto-released with "release_read_only"), prepared inputs
//   taken by token, Push matched to the batch's outputs by feature id,
//   a frozen Save / Resume / ReadCheckpoint cycle, Join, Close, Abort.
// The gather, pooling, coalescing and LazyAdam all run in the store's kernels;
// padding keys are dropped on the device (the adapter's PrepareAdapterInput).
//
// The configuration is JSON; a small parser for the subset the configuration
// uses (objects, arrays, strings, numbers with exact 64-bit integers, booleans,
// null) is included, since the reference's JSON library is not a dependency of
// this build.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <optional>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

#include "eps_b200.h"
#include "eps_b200_runtime_c.h"

namespace {

struct Fail : std::runtime_error {
  int code;
  Fail(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};
void Require(bool ok, const std::string& m, int code = EPS_B200_INVALID_ARGUMENT) {
  if (!ok) throw Fail(code, m);
}
void Call(int rc, const EpsB200Status& st) {
  if (rc) throw Fail(rc, st.message);
}

// adapters/entropy/runtime_c.cpp:20-29: 0 or Error::Code + 1 with the message
template <typename F>
int Boundary(EpsStatus* status, F fn) noexcept {
  if (status) { status->code = 0; status->message[0] = 0; }
  auto fail = [&](int code, const char* m) {
    if (status) {
      status->code = code;
      std::strncpy(status->message, m, sizeof(status->message) - 1);
      status->message[sizeof(status->message) - 1] = 0;
    }
    return code;
  };
  try { fn(); return 0; }
  catch (const Fail& e) { return fail(e.code, e.what()); }
  catch (const std::bad_alloc&) { return fail(EPS_B200_CAPACITY_EXCEEDED, "native runtime allocation failed"); }
  catch (const std::exception& e) { return fail(EPS_B200_RUN_FAILED, e.what()); }
  catch (...) { return fail(EPS_B200_RUN_FAILED, "unknown native runtime failure"); }
}

// ------------------------------------------------------------------- JSON
struct Json {
  enum Kind { kNull, kBool, kNumber, kString, kArray, kObject } kind = kNull;
  bool b = false;
  double num = 0;
  bool integral = false, negative = false;
  uint64_t u = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;

  bool Has(const std::string& k) const {
    if (kind != kObject) return false;
    for (auto& kv : obj) if (kv.first == k) return true;
    return false;
  }
  const Json& At(const std::string& k) const {
    Require(kind == kObject, "JSON object expected");
    for (auto& kv : obj) if (kv.first == k) return kv.second;
    throw Fail(EPS_B200_INVALID_ARGUMENT, "missing JSON field '" + k + "'");
  }
  double Num() const { Require(kind == kNumber, "JSON number expected"); return num; }
  uint64_t U64() const {
    Require(kind == kNumber && integral && !negative, "JSON unsigned integer expected");
    return u;
  }
  uint32_t U32() const {
    const uint64_t v = U64();
    Require(v <= 0xFFFFFFFFull, "JSON integer out of range");
    return (uint32_t)v;
  }
  const std::string& Str() const { Require(kind == kString, "JSON string expected"); return str; }
  bool Bool() const { Require(kind == kBool, "JSON boolean expected"); return b; }
  uint64_t U64Or(const std::string& k, uint64_t d) const { return Has(k) ? At(k).U64() : d; }
  std::string StrOr(const std::string& k, const std::string& d) const { return Has(k) ? At(k).Str() : d; }
  bool BoolOr(const std::string& k, bool d) const { return Has(k) ? At(k).Bool() : d; }
};

struct Parser {
  const char* p;
  const char* end;
  void Ws() { while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p; }
  char Peek() { Ws(); Require(p < end, "truncated JSON"); return *p; }
  void Expect(char c) { Require(Peek() == c, std::string("JSON: expected '") + c + "'"); ++p; }
  bool Literal(const char* w) {
    const size_t n = std::strlen(w);
    if ((size_t)(end - p) >= n && std::strncmp(p, w, n) == 0) { p += n; return true; }
    return false;
  }
  static void Utf8(std::string& out, unsigned v) {
    if (v < 0x80) out += (char)v;
    else if (v < 0x800) { out += (char)(0xC0 | (v >> 6)); out += (char)(0x80 | (v & 63)); }
    else if (v < 0x10000) {
      out += (char)(0xE0 | (v >> 12)); out += (char)(0x80 | ((v >> 6) & 63)); out += (char)(0x80 | (v & 63));
    } else {
      out += (char)(0xF0 | (v >> 18)); out += (char)(0x80 | ((v >> 12) & 63));
      out += (char)(0x80 | ((v >> 6) & 63)); out += (char)(0x80 | (v & 63));
    }
  }
  unsigned Hex4() {
    Require(end - p >= 4, "truncated JSON escape");
    unsigned v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (unsigned)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (unsigned)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (unsigned)(c - 'A' + 10);
      else throw Fail(EPS_B200_INVALID_ARGUMENT, "invalid JSON escape");
    }
    return v;
  }
  std::string String() {
    Expect('"');
    std::string out;
    while (true) {
      Require(p < end, "truncated JSON string");
      char c = *p++;
      if (c == '"') break;
      Require((unsigned char)c >= 0x20, "control character in JSON string");
      if (c != '\\') { out += c; continue; }
      Require(p < end, "truncated JSON escape");
      c = *p++;
      switch (c) {
        case '"': case '\\': case '/': out += c; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          unsigned v = Hex4();
          if (v >= 0xD800 && v < 0xDC00 && end - p >= 6 && p[0] == '\\' && p[1] == 'u') {
            p += 2;
            const unsigned lo = Hex4();
            Require(lo >= 0xDC00 && lo < 0xE000, "invalid JSON surrogate pair");
            v = 0x10000 + ((v - 0xD800) << 10) + (lo - 0xDC00);
          }
          Utf8(out, v);
          break;
        }
        default: throw Fail(EPS_B200_INVALID_ARGUMENT, "invalid JSON escape");
      }
    }
    return out;
  }
  Json Value(int depth = 0) {
    Require(depth < 64, "JSON nesting too deep");
    Json v;
    const char c = Peek();
    if (c == '{') {
      ++p;
      v.kind = Json::kObject;
      if (Peek() == '}') { ++p; return v; }
      while (true) {
        std::string k = String();
        Expect(':');
        v.obj.emplace_back(std::move(k), Value(depth + 1));
        if (Peek() == ',') { ++p; continue; }
        Expect('}');
        return v;
      }
    }
    if (c == '[') {
      ++p;
      v.kind = Json::kArray;
      if (Peek() == ']') { ++p; return v; }
      while (true) {
        v.arr.push_back(Value(depth + 1));
        if (Peek() == ',') { ++p; continue; }
        Expect(']');
        return v;
      }
    }
    if (c == '"') { v.kind = Json::kString; v.str = String(); return v; }
    if (Literal("true")) { v.kind = Json::kBool; v.b = true; return v; }
    if (Literal("false")) { v.kind = Json::kBool; v.b = false; return v; }
    if (Literal("null")) return v;
    // number: exact unsigned integers, otherwise a double
    const char* s = p;
    if (p < end && *p == '-') ++p;
    bool integral = true;
    while (p < end && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' ||
                       ((*p == '-' || *p == '+') && (p[-1] == 'e' || p[-1] == 'E')))) {
      if (*p == '.' || *p == 'e' || *p == 'E') integral = false;
      ++p;
    }
    Require(p > s && (p[-1] >= '0' && p[-1] <= '9'), "invalid JSON value");
    const std::string text(s, p);
    char* stop = nullptr;
    v.kind = Json::kNumber;
    v.num = std::strtod(text.c_str(), &stop);
    Require(stop && *stop == 0, "invalid JSON number");
    v.negative = text[0] == '-';
    if (integral && !v.negative) {
      errno = 0;
      v.u = std::strtoull(text.c_str(), nullptr, 10);
      v.integral = errno == 0;
    }
    return v;
  }
};

// adapters/entropy/runtime_c.cpp:30: at most 1 MiB of JSON
Json Parse(const char* text) {
  Require(text != nullptr && strnlen(text, (1 << 20) + 1) <= (1u << 20), "native JSON exceeds limit");
  Parser ps{text, text + std::strlen(text)};
  Json v = ps.Value();
  ps.Ws();
  Require(ps.p == ps.end, "trailing JSON data");
  return v;
}

std::string Quote(const std::string& s) {
  std::string o = "\"";
  for (unsigned char c : s) {
    if (c == '"' || c == '\\') { o += '\\'; o += (char)c; }
    else if (c < 0x20) { char b[8]; std::snprintf(b, sizeof(b), "\\u%04x", c); o += b; }
    else o += (char)c;
  }
  return o + "\"";
}
std::string Bool(bool v) { return v ? "true" : "false"; }

// adapters/entropy/runtime_c.cpp:31-35: lower-case hex of checkpoint bytes
std::string Hex(const std::string& data) {
  static const char digits[] = "0123456789abcdef";
  std::string out;
  for (unsigned char c : data) { out += digits[c >> 4]; out += digits[c & 15]; }
  return out;
}
std::string Unhex(const std::string& text) {
  Require(text.size() <= 16 && text.size() % 2 == 0, "invalid checksum tail");
  auto digit = [](char c) {
    Require((c >= '0' && c <= '9') || (c >= 'a' && c <= 'f'), "invalid checksum tail");
    return c <= '9' ? c - '0' : c - 'a' + 10;
  };
  std::string out;
  for (size_t i = 0; i < text.size(); i += 2) out += (char)((digit(text[i]) << 4) | digit(text[i + 1]));
  return out;
}

// adapters/entropy/runtime_c.cpp:36-41: a float32 sparse LazyAdam table
EpsB200Table TableOf(const Json& t, uint64_t epoch) {
  Require(t.StrOr("dtype", "float32") == "float32" &&
          t.At("optimizer").At("kind").Str() == "sparse_lazy_adam", "unsupported native table format");
  const Json& o = t.At("optimizer");
  const Json& i = t.At("initialization");
  EpsB200Table d{};
  d.id = t.At("id").U32();
  d.dimension = t.At("dimension").U32();
  d.shard_count = 1;
  d.partition_epoch = epoch;
  d.learning_rate = (float)o.At("learning_rate").Num();
  d.beta1 = (float)o.At("beta1").Num();
  d.beta2 = (float)o.At("beta2").Num();
  d.epsilon = (float)o.At("epsilon").Num();
  d.initial_beta1_power = (float)o.At("initial_beta1_power").Num();
  d.initial_beta2_power = (float)o.At("initial_beta2_power").Num();
  if (o.Has("weight_bounds")) {
    const Json& b = o.At("weight_bounds");
    Require(b.kind == Json::kArray && b.arr.size() == 2, "invalid weight bounds");
    d.has_weight_bounds = 1;
    d.weight_min = (float)b.arr[0].Num();
    d.weight_max = (float)b.arr[1].Num();
  }
  d.initialization_min = (float)i.At("min").Num();
  d.initialization_max = (float)i.At("max").Num();
  d.initialization_seed = i.At("seed").U64();
  // "key_space": a dense table of keys [0, key_space); without it (the reference's
  // own table JSON) a hashed table of any 64-bit keys, "capacity" rows (default
  // 2^20) created on first touch
  if (t.Has("key_space")) {
    d.key_space = t.At("key_space").U64();
  } else {
    d.key_space = 0;
    d.capacity = t.Has("capacity") ? t.At("capacity").U64() : (1ull << 20);
  }
  return d;
}

void MakeDirs(const std::string& dir) {
  for (size_t pos = 1; pos <= dir.size(); ++pos) {
    if (pos < dir.size() && dir[pos] != '/') continue;
    const std::string part = dir.substr(0, pos);
    if (::mkdir(part.c_str(), 0755) != 0 && errno != EEXIST)
      throw Fail(EPS_B200_UNAVAILABLE, "cannot create snapshot directory " + part);
  }
}

// ------------------------------------------------------------- ownership
struct DeviceBlock {             // one allocation for a batch's device outputs
  void* data = nullptr;
  int device = -1;
  ~DeviceBlock() {
    if (data) { cudaSetDevice(device); cudaFree(data); }
  }
};
struct BufferOwner {
  std::vector<float> host;
  std::shared_ptr<DeviceBlock> device;
};
void ReleaseBuffer(void* p) { delete static_cast<BufferOwner*>(p); }
// The pull is complete when it returns (host inputs make the store's lookup
// synchronous), so a consumer stream needs no extra dependency.
int WaitBuffer(void*, void*, EpsStatus* status) { return Boundary(status, [] {}); }
struct BatchOwner {
  std::vector<EpsBuffer> buffers;
  ~BatchOwner() { for (auto& b : buffers) if (b.owner) b.release(b.owner); }
};
void ReleaseBatch(void* p) { delete static_cast<BatchOwner*>(p); }
void ReleaseText(void* p) { delete static_cast<std::string*>(p); }

// ------------------------------------------------------------------ batches
struct Input {                   // owned copy of one request's features
  std::vector<std::vector<uint64_t>> keys, offsets;
  std::vector<EpsB200Feature> feats;
};
struct Output { uint32_t feature; uint64_t rows, columns; };
struct Batch {
  uint64_t ticket = UINT64_MAX;  // the store's lookup ticket (none when read-only)
  bool read_only = false;
  std::vector<Output> outputs;
};

constexpr uint64_t kCompletionHistory = 4096;   // AdapterOptions::completion_history
constexpr uint64_t kMaxPending = 8;             // PreparationOptions::max_pending_batches

struct Runtime {
  std::mutex mutex;
  EpsB200Store* store = nullptr;
  int device = 0;
  std::string run, snapshot_dir;
  uint64_t epoch = 1, max_live = 128;
  bool release_read_only = false;
  std::map<uint32_t, uint32_t> dims;
  std::map<uint32_t, bool> prediction;           // table_mode
  // adapter lifecycle (adapters/entropy/table_adapter.cpp:100-104)
  std::map<uint64_t, Batch> live;
  std::map<uint64_t, bool> completed;
  uint64_t next = 0;
  bool closed = false;                           // adapter input closed (frozen save or failure)
  std::optional<std::string> saved, resumed;
  std::map<uint64_t, Input> prepared;
  uint64_t next_token = 0;
  // RestoredSnapshot (include/eps/types.hpp:41-48) of a "restore" at create
  bool loaded = false, pristine = false;
  std::string source_run;
  uint64_t restored_bytes = 0, restored_checksum = 0;

  ~Runtime() { Close(); }
  void Close() {
    if (store) eps_b200_destroy(store);
    store = nullptr;
  }
  void Ready() { Require(store != nullptr, "native runtime is closed", EPS_B200_UNAVAILABLE); }
  void AdapterReady() {          // table_adapter.cpp:42-45
    Require(!closed, "adapter input is closed", EPS_B200_UNAVAILABLE);
    Require(live.size() < max_live, "adapter live-batch limit reached", EPS_B200_CAPACITY_EXCEEDED);
  }
  void CreateTable(const Json& t) {
    Require(!closed, "adapter input is closed", EPS_B200_UNAVAILABLE);
    EpsB200Table d = TableOf(t, epoch);
    const bool existed = dims.count(d.id) != 0;
    EpsB200Status st;
    Call(eps_b200_create_table(store, &d, &st), st);
    dims[d.id] = d.dimension;
    if (!existed) pristine = false;
  }
  // runtime_c.cpp:83-87: prediction tables make a batch read-only; no mixing
  bool ReadOnly(const Input& in, bool requested) const {
    if (requested) return true;
    bool any = false, all = true;
    for (const auto& f : in.feats) {
      auto it = prediction.find(f.table);
      const bool v = it != prediction.end() && it->second;
      any |= v;
      all &= v;
    }
    Require(!any || all, "native batch mixes training and prediction tables");
    return any;
  }
  void Finish(uint64_t handle, bool pushed) {    // table_adapter.cpp:33-41
    completed.at(handle) = pushed;
    live.erase(handle);
    while (completed.size() > kCompletionHistory) {
      auto it = completed.begin();
      while (it != completed.end() && live.count(it->first)) ++it;
      if (it == completed.end()) break;
      completed.erase(it);
    }
  }
};

Runtime& Get(void* p) {
  Require(p != nullptr, "null native runtime");
  return *static_cast<Runtime*>(p);
}

// runtime_c.cpp:135-146 (limits of the native input) and the adapter's
// preparation checks (src/access/prepare_queue.cpp:21-33).
Input Copy(const EpsFeature* in, uint64_t count) {
  Require(in && count > 0 && count <= 1024, "invalid native feature count");
  Input f;
  f.keys.resize(count);
  f.offsets.resize(count);
  f.feats.resize(count);
  uint64_t bytes = 0;
  std::set<uint32_t> ids;
  for (uint64_t i = 0; i < count; ++i) {
    const auto& x = in[i];
    Require(x.pooling <= 2 && x.key_count <= (16ull << 20) / 8 && x.offset_count <= (16ull << 20) / 8 &&
            (!x.key_count || x.keys) && x.offset_count && x.offsets, "invalid native feature input");
    bytes += (x.key_count + x.offset_count) * 8;
    Require(bytes <= (16ull << 20), "native feature input exceeds budget");
    f.keys[i].assign(x.keys, x.keys + x.key_count);
    f.offsets[i].assign(x.offsets, x.offsets + x.offset_count);
    Require(ids.insert(x.feature).second, "duplicate adapter feature");
    const auto& o = f.offsets[i];
    bool sorted = true;
    for (size_t j = 1; j < o.size(); ++j) sorted &= o[j - 1] <= o[j];
    Require(o.front() == 0 && o.back() == x.key_count && sorted, "invalid adapter row splits");
    EpsB200Feature& g = f.feats[i];
    g = EpsB200Feature{};
    g.table = x.table;
    g.feature = x.feature;
    g.pooling = x.pooling;
    g.has_padding = x.has_padding ? 1u : 0u;
    g.padding_key = x.padding_key;
    g.keys = f.keys[i].data();
    g.key_count = x.key_count;
    g.offsets = f.offsets[i].data();
    g.offset_count = x.offset_count;
  }
  return f;
}

// The adapter's Dispatch (table_adapter.cpp:46-92) + runtime_c.cpp's Pack and
// Publish (runtime_c.cpp:160-178): outputs in feature order, sequence features
// [key_count, dim] with padding positions zero.
void Dispatch(Runtime& r, Input& in, bool read_only, bool device, EpsBatch* output) {
  Require(r.next != UINT64_MAX, "adapter request sequence exhausted", EPS_B200_CAPACITY_EXCEEDED);
  const uint64_t n = in.feats.size();
  std::vector<Output> shapes(n);
  uint64_t total = 0;
  for (uint64_t i = 0; i < n; ++i) {
    const auto& f = in.feats[i];
    auto it = r.dims.find(f.table);
    Require(it != r.dims.end(), "unknown table");
    shapes[i] = Output{f.feature, f.pooling == EPS_B200_SEQUENCE ? f.key_count : f.offset_count - 1, it->second};
    total += shapes[i].rows * shapes[i].columns;
  }
  auto owner = std::make_unique<BatchOwner>();
  owner->buffers.reserve(n);
  std::vector<EpsB200Buffer> outs(n);
  std::shared_ptr<DeviceBlock> block;
  if (device) {
    block = std::make_shared<DeviceBlock>();
    Require(cudaSetDevice(r.device) == cudaSuccess, "cudaSetDevice failed", EPS_B200_RUN_FAILED);
    const cudaError_t e = cudaMalloc(&block->data, std::max<uint64_t>(total * 4, 256));
    Require(e == cudaSuccess, cudaGetErrorString(e),
            e == cudaErrorMemoryAllocation ? EPS_B200_CAPACITY_EXCEEDED : EPS_B200_RUN_FAILED);
    block->device = r.device;
  }
  uint64_t at = 0;
  for (uint64_t i = 0; i < n; ++i) {
    auto b = std::make_unique<BufferOwner>();
    void* data;
    const uint64_t values = shapes[i].rows * shapes[i].columns;
    if (device) {
      b->device = block;
      data = static_cast<float*>(block->data) + at;
      at += values;
    } else {
      b->host.resize(values);
      data = b->host.data();
    }
    outs[i] = EpsB200Buffer{shapes[i].feature, 0, shapes[i].rows, shapes[i].columns, data,
                            device ? r.device : -1, 0};
    owner->buffers.push_back(EpsBuffer{shapes[i].feature, shapes[i].rows, shapes[i].columns, data,
                                       device ? r.device : -1, b.get(), ReleaseBuffer, WaitBuffer});
    b.release();
  }
  Batch batch;
  batch.read_only = read_only;
  batch.outputs = shapes;
  EpsB200Status st;
  // host inputs make the lookup synchronous: outputs are complete on return
  Call(eps_b200_lookup(r.store, in.feats.data(), n, 0, read_only, 0, outs.data(), nullptr,
                       read_only ? nullptr : &batch.ticket, &st), st);
  r.pristine = false;
  const uint64_t handle = r.next++;
  r.completed.emplace(handle, false);
  r.live.emplace(handle, std::move(batch));
  uint64_t published = handle;
  if (read_only && r.release_read_only) {
    r.Finish(handle, false);
    published = UINT64_MAX;
  }
  *output = EpsBatch{published, owner->buffers.size(), owner->buffers.data(), owner.get(), ReleaseBatch};
  owner.release();
}

// ------------------------------------------------------------ entry points
int Create(const char* text, void** output, EpsStatus* status) {
  if (output) *output = nullptr;
  return Boundary(status, [&] {
    Require(output != nullptr, "null runtime output");
    const Json c = Parse(text);
    Require(c.kind == Json::kObject, "native configuration must be a JSON object");
    Require(!c.Has("agents") && !c.Has("cuda") && !c.Has("training"),
            "agents, cuda and training sections are not supported by the B200 runtime");
    auto r = std::make_unique<Runtime>();
    r->run = c.At("run").Str();
    r->epoch = c.U64Or("epoch", 1);
    r->device = (int)c.U64Or("device", 0);
    r->max_live = c.U64Or("max_live", 128);
    Require(r->max_live > 0 && r->max_live <= (1u << 20), "invalid native live-batch limit");
    r->release_read_only = c.BoolOr("release_read_only", false);
    r->snapshot_dir = c.StrOr("snapshot_directory", "snapshots");
    Require(c.At("tables").kind == Json::kArray, "native tables must be a JSON array");
    EpsB200Options o{};
    o.device = r->device;
    o.shard_id = 0;
    o.shard_count = 1;
    o.max_live_tickets = (uint32_t)r->max_live;
    o.partition_epoch = r->epoch;
    o.state_bytes = c.U64Or("state_bytes", 64ull << 30);
    EpsB200Status st;
    Call(eps_b200_create(&o, &r->store, &st), st);
    for (const auto& t : c.At("tables").arr) r->CreateTable(t);
    if (c.Has("restore")) {      // eps_server --restore (src/server/main.cpp:89-90)
      const std::string path = c.At("restore").Str();
      EpsB200SnapshotInfo info{};
      Call(eps_b200_snapshot_inspect(path.c_str(), &info, nullptr, 0, &st), st);
      Call(eps_b200_snapshot_read(r->store, path.c_str(), r->run.c_str(), &st), st);
      struct stat sb{};
      Require(::stat(path.c_str(), &sb) == 0, "cannot stat snapshot", EPS_B200_UNAVAILABLE);
      r->loaded = r->pristine = true;
      r->source_run = info.run;
      r->restored_bytes = (uint64_t)sb.st_size;
      r->restored_checksum = info.checksum;
    }
    *output = r.release();
  });
}

void Destroy(void* p) {
  try { delete static_cast<Runtime*>(p); } catch (...) {}
}

int Pull(void* p, const EpsFeature* features, uint64_t count, int32_t read_only, int32_t device,
         EpsBatch* output, EpsStatus* status) {
  if (output) *output = EpsBatch{};
  return Boundary(status, [&] {
    Require(output != nullptr, "null batch output");
    auto& r = Get(p);
    std::lock_guard<std::mutex> lock(r.mutex);
    r.Ready();
    Input in = Copy(features, count);
    const bool mode = r.ReadOnly(in, read_only != 0);
    r.AdapterReady();
    Require(r.prepared.empty(), "consume or cancel prepared inputs before synchronous Pull",
            EPS_B200_UNAVAILABLE);
    Dispatch(r, in, mode, device != 0, output);
  });
}

int Prepare(void* p, const EpsFeature* features, uint64_t count, uint64_t* token, EpsStatus* status) {
  return Boundary(status, [&] {
    Require(token != nullptr, "null token output");
    auto& r = Get(p);
    std::lock_guard<std::mutex> lock(r.mutex);
    r.Ready();
    Input in = Copy(features, count);
    // src/access/prepare_queue.cpp:120-132
    Require(!r.closed, "preparation admission is closed", EPS_B200_UNAVAILABLE);
    Require(r.next_token != UINT64_MAX && r.prepared.size() < kMaxPending, "preparation queue is full",
            EPS_B200_CAPACITY_EXCEEDED);
    *token = r.next_token++;
    r.prepared.emplace(*token, std::move(in));
  });
}

int PullPrepared(void* p, uint64_t token, int32_t read_only, int32_t device, EpsBatch* output,
                 EpsStatus* status) {
  if (output) *output = EpsBatch{};
  return Boundary(status, [&] {
    Require(output != nullptr, "null prepared output");
    auto& r = Get(p);
    std::lock_guard<std::mutex> lock(r.mutex);
    r.Ready();
    auto it = r.prepared.find(token);
    Require(it != r.prepared.end(), "unknown native prepared token");
    Input in = std::move(it->second);
    r.prepared.erase(it);         // consumed whatever the outcome (runtime_c.cpp:196)
    const bool mode = r.ReadOnly(in, read_only != 0);
    r.AdapterReady();
    Dispatch(r, in, mode, device != 0, output);
  });
}

int Push(void* p, uint64_t handle, const EpsBuffer* input, uint64_t count, void* stream,
         EpsStatus* status) {
  return Boundary(status, [&] {
    auto& r = Get(p);
    std::lock_guard<std::mutex> lock(r.mutex);
    r.Ready();
    Require(input && count > 0 && count <= 1024, "invalid native gradient count");
    uint64_t bytes = 0;
    for (uint64_t i = 0; i < count; ++i) {
      const auto& b = input[i];
      // runtime_c.cpp:203-205: shape and 64 MiB budget
      Require(b.columns > 0 && b.columns <= (64ull << 20) / 4 && b.rows <= (64ull << 20) / (4 * b.columns),
              "invalid native gradient shape");
      bytes += b.rows * b.columns * 4;
      Require(bytes <= (64ull << 20) && (!(b.rows * b.columns) || b.data),
              "native gradient budget/pointer invalid");
      Require(b.device < 0 || b.device == r.device, "gradient device mismatch");
    }
    // table_adapter.cpp:163-185: match the batch's outputs by feature id
    auto live = r.live.find(handle);
    if (live == r.live.end()) {
      auto c = r.completed.find(handle);
      Require(c != r.completed.end() && c->second, "unknown or released adapter batch",
              EPS_B200_RETIRED_REQUEST);
      return;
    }
    const Batch& batch = live->second;
    Require(!batch.read_only && count == batch.outputs.size(), "invalid adapter Push");
    std::map<uint32_t, const EpsBuffer*> by_id;
    for (uint64_t i = 0; i < count; ++i)
      Require(by_id.emplace(input[i].feature, &input[i]).second, "duplicate gradient feature");
    std::vector<EpsB200Buffer> g(count);
    for (uint64_t i = 0; i < count; ++i) {
      const Output& o = batch.outputs[i];
      auto it = by_id.find(o.feature);
      Require(it != by_id.end(), "missing adapter gradient");
      const EpsBuffer& b = *it->second;
      Require(b.rows == o.rows && b.columns == o.columns, "adapter gradient shape mismatch");
      g[i] = EpsB200Buffer{b.feature, 0, b.rows, b.columns, b.data, b.device < 0 ? -1 : b.device, 0};
    }
    EpsB200Status st;
    const int rc = eps_b200_push(r.store, batch.ticket, g.data(), count, stream, 1, &st);
    if (rc) {                     // table_adapter.cpp:186-188: admission closes
      r.closed = true;
      throw Fail(rc, st.message);
    }
    r.Finish(handle, true);
  });
}

// ReadSnapshotChunk (src/store/snapshot.cpp:138-157) + the checksum
// continuation of runtime_c.cpp:256-266.
std::string ReadCheckpoint(Runtime& r, const Json& args) {
  const std::string id = args.At("id").Str();
  const uint64_t shard = args.At("shard").U64();
  const uint64_t offset = args.At("offset").U64();
  const uint64_t max_bytes = args.At("max_bytes").U64();
  uint64_t checksum = args.At("checksum").U64();
  const std::string tail = Unhex(args.At("tail").Str());
  Require(tail.size() == std::min<uint64_t>(offset, 8) && (offset || checksum == 14695981039346656037ull),
          "invalid checkpoint checksum continuation");
  Require(r.closed && r.saved && *r.saved == id, "export requires the adapter's successful frozen save",
          EPS_B200_UNAVAILABLE);
  Require(shard < 1, "checkpoint shard is out of range");
  Require(max_bytes > 0 && max_bytes <= (1u << 20), "checkpoint chunk exceeds 1 MiB limit");
  const std::string path = r.snapshot_dir + "/" + id + "/shard-0.bin";
  const int fd = ::open(path.c_str(), O_RDONLY);
  Require(fd >= 0, "cannot open checkpoint", EPS_B200_UNAVAILABLE);
  std::string data;
  uint64_t size = 0;
  try {
    struct stat info{};
    Require(::fstat(fd, &info) == 0 && S_ISREG(info.st_mode) && info.st_size >= 8, "invalid checkpoint file",
            EPS_B200_UNAVAILABLE);
    size = (uint64_t)info.st_size;
    Require(offset <= size, "checkpoint offset exceeds file size");
    data.resize(std::min<uint64_t>(max_bytes, size - offset));
    for (size_t done = 0; done < data.size();) {
      const ssize_t n = ::pread(fd, &data[done], data.size() - done, (off_t)(offset + done));
      if (n < 0 && errno == EINTR) continue;
      Require(n > 0, "checkpoint file changed during export", EPS_B200_UNAVAILABLE);
      done += (size_t)n;
    }
  } catch (...) {
    ::close(fd);
    throw;
  }
  ::close(fd);
  const bool eof = offset + data.size() == size;
  const std::string combined = tail + data;
  const size_t body = combined.size() > 8 ? combined.size() - 8 : 0;
  for (size_t i = 0; i < body; ++i) checksum = (checksum ^ (unsigned char)combined[i]) * 1099511628211ull;
  const std::string next_tail = combined.substr(body);
  if (eof) {
    Require(next_tail.size() == 8, "checkpoint checksum trailer missing");
    uint64_t expected = 0;
    for (unsigned i = 0; i < 8; ++i) expected |= (uint64_t)(unsigned char)next_tail[i] << (8 * i);
    Require(expected == checksum, "exported checkpoint checksum mismatch", EPS_B200_RUN_FAILED);
  }
  return "{\"offset\":" + std::to_string(offset) + ",\"total_bytes\":" + std::to_string(size) +
         ",\"data\":\"" + Hex(data) + "\",\"eof\":" + Bool(eof) + ",\"checksum\":" + std::to_string(checksum) +
         ",\"tail\":\"" + Hex(next_tail) + "\"}";
}

int Command(void* p, const char* command, const char* arguments, EpsText* output, EpsStatus* status) {
  if (output) *output = EpsText{};
  return Boundary(status, [&] {
    Require(command && output, "invalid native control output");
    auto& r = Get(p);
    std::lock_guard<std::mutex> lock(r.mutex);
    r.Ready();
    const Json args = Parse(arguments);
    const std::string method(command);
    std::string result = "null";
    EpsB200Status st;
    if (method == "join") {
      Require(r.live.empty(), "complete Push/Release before Join", EPS_B200_UNAVAILABLE);
      Call(eps_b200_synchronize(r.store, &st), st);
    } else if (method.rfind("training_", 0) == 0) {
      // runtime_c.cpp:213-248: this runtime has no training coordinator
      Require(false, "native training is not configured");
    } else if (method == "create_table") {
      r.CreateTable(args);
    } else if (method == "release") {
      const uint64_t handle = args.At("handle").U64();
      auto it = r.live.find(handle);
      if (it == r.live.end()) {
        Require(r.completed.count(handle) != 0, "retired adapter batch", EPS_B200_RETIRED_REQUEST);
      } else {
        if (it->second.ticket != UINT64_MAX) Call(eps_b200_release(r.store, it->second.ticket, &st), st);
        r.Finish(handle, false);
      }
    } else if (method == "cancel_prepared") {
      const uint64_t token = args.At("token").U64();
      Require(r.prepared.erase(token) == 1, "unknown or consumed preparation token", EPS_B200_RETIRED_REQUEST);
    } else if (method == "table_mode") {
      Require(r.release_read_only, "table modes require automatic read-only release");
      Require(r.live.empty(), "complete Push/Release before Join", EPS_B200_UNAVAILABLE);
      r.prediction[args.At("table").U32()] = args.At("prediction").Bool();
    } else if (method == "save") {
      // TableAdapter::Save (table_adapter.cpp:230-245) over DrainAndFlush
      // (src/server/service.cpp:588-621)
      const std::string id = args.At("id").Str();
      bool ok = !id.empty() && id.size() <= 128 && id != "." && id != "..";
      for (unsigned char c : id)
        ok = ok && ((c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || (c >= '0' && c <= '9') || c == '_' ||
                    c == '-' || c == '.');
      Require(!r.closed, "adapter input is closed", EPS_B200_UNAVAILABLE);
      Require(r.live.empty(), "complete all batches before saving", EPS_B200_UNAVAILABLE);
      Require(r.prepared.empty(), "consume or cancel prepared inputs before saving", EPS_B200_UNAVAILABLE);
      r.closed = true;
      r.saved.reset();
      r.resumed.reset();
      Require(ok, "invalid snapshot ID");
      const std::string dir = r.snapshot_dir + "/" + id;
      const std::string path = dir + "/shard-0.bin";
      MakeDirs(dir);
      Call(eps_b200_synchronize(r.store, &st), st);
      Call(eps_b200_snapshot_write(r.store, path.c_str(), r.run.c_str(), 0, &st), st);
      r.saved = id;
      result = "[" + Quote(path) + "]";
    } else if (method == "resume") {
      // TableAdapter::Resume (table_adapter.cpp:257-271)
      const std::string id = args.At("id").Str();
      if (!(!r.closed && r.resumed && *r.resumed == id)) {
        Require(r.closed && r.saved && *r.saved == id, "resume requires the adapter's successful frozen save",
                EPS_B200_UNAVAILABLE);
        r.resumed = id;
        r.saved.reset();
        r.closed = false;
      }
    } else if (method == "read_checkpoint") {
      result = ReadCheckpoint(r, args);
    } else if (method == "endpoint") {
      result = "\"\"";
    } else if (method == "restored_from") {
      result = "[{\"loaded\":" + Bool(r.loaded) + ",\"pristine\":" + Bool(r.pristine) + ",\"run\":" +
               Quote(r.run) + ",\"source_run\":" + Quote(r.source_run) + ",\"bytes\":" +
               std::to_string(r.restored_bytes) + ",\"checksum\":" + std::to_string(r.restored_checksum) +
               ",\"shard\":0,\"shard_count\":1,\"partition_epoch\":" + std::to_string(r.epoch) + "}]";
    } else if (method == "stats") {
      EpsB200Stats s{};
      Call(eps_b200_stats(r.store, &s, &st), st);
      // cached_rows: rows held on a GPU, which is every row of this store
      result = "[{\"updates\":" + std::to_string(s.updates) + ",\"live_tickets\":" +
               std::to_string(s.live_tickets) + ",\"cached_rows\":" + std::to_string(s.rows) + "}]";
    } else if (method == "close") {
      Require(r.live.empty(), "complete Push/Release before Join", EPS_B200_UNAVAILABLE);
      Call(eps_b200_synchronize(r.store, &st), st);
      r.Close();
    } else if (method == "abort") {
      r.Close();
    } else {
      Require(false, "unknown native control command");
    }
    auto owner = std::make_unique<std::string>(result);
    *output = EpsText{owner->data(), owner->size(), owner.get(), ReleaseText};
    owner.release();
  });
}

const EpsRuntimeApi kApi{EPS_RUNTIME_ABI, sizeof(EpsRuntimeApi), Create, Destroy, Pull, Prepare,
                         PullPrepared, Push, Command};

}  // namespace

extern "C" EPS_RUNTIME_EXPORT const EpsRuntimeApi* eps_runtime_api_v1(void) { return &kApi; }
