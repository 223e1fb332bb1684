// Model files and training-state files (host side): formats and the
// reference functions each entry replaces are in include/llmk_gpt2.h.
// Everything goes through the public model calls (load / read parameters and
// optimizer moments), so the files always hold llm.c parameter order.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "llmk_gpt2.h"
#include "runtime.h"

using llmk::fail;

namespace {

constexpr int kHeaderInts = 256;
constexpr int32_t kModelMagic = 20240326, kModelVersion = 3;
constexpr int32_t kStateMagic = 20241202, kStateVersion = 1;

void put_config(int32_t* h, const llmk_gpt2_config& c) {
  h[2] = c.max_seq_len;
  h[3] = c.vocab_size;
  h[4] = c.num_layers;
  h[5] = c.num_heads;
  h[6] = c.channels;
  h[7] = c.padded_vocab_size;
}

llmk_gpt2_config get_config(const int32_t* h) {
  llmk_gpt2_config c;
  c.max_seq_len = h[2];
  c.vocab_size = h[3];
  c.num_layers = h[4];
  c.num_heads = h[5];
  c.channels = h[6];
  c.padded_vocab_size = h[7];
  return c;
}

bool same_config(const llmk_gpt2_config& a, const llmk_gpt2_config& b) {
  return a.max_seq_len == b.max_seq_len && a.vocab_size == b.vocab_size && a.padded_vocab_size == b.padded_vocab_size &&
         a.num_layers == b.num_layers && a.num_heads == b.num_heads && a.channels == b.channels;
}

bool plausible(const llmk_gpt2_config& c) {
  return c.max_seq_len > 0 && c.vocab_size > 0 && c.padded_vocab_size >= c.vocab_size && c.num_layers > 0 &&
         c.num_heads > 0 && c.channels > 0 && c.channels % c.num_heads == 0;
}

// Opens `path`, reads and validates the header (magic, version, a plausible
// configuration, file size == header + sections * nparams fp32 values).
int open_checked(std::ifstream& f, const char* path, int32_t magic, int32_t version, int sections, int32_t* h,
                 llmk_gpt2_config* cfg, size_t* nparams) {
  if (!path) return fail(LLMK_ERR_INVALID_ARG, "checkpoint: null path");
  f.open(path, std::ios::binary);
  if (!f.is_open()) return fail(LLMK_ERR_INVALID_ARG, std::string("checkpoint: cannot open ") + path);
  if (!f.read(reinterpret_cast<char*>(h), kHeaderInts * sizeof(int32_t)))
    return fail(LLMK_ERR_INVALID_ARG, std::string("checkpoint: cannot read the header of ") + path);
  if (h[0] != magic) return fail(LLMK_ERR_INVALID_ARG, std::string("checkpoint: bad magic in ") + path);
  if (h[1] != version) return fail(LLMK_ERR_INVALID_ARG, std::string("checkpoint: bad version in ") + path);
  *cfg = get_config(h);
  if (!plausible(*cfg)) return fail(LLMK_ERR_INVALID_ARG, std::string("checkpoint: bad configuration in ") + path);
  *nparams = llmk_gpt2_num_parameters(cfg);
  f.seekg(0, std::ios::end);
  const long long size = static_cast<long long>(f.tellg());
  f.seekg(kHeaderInts * sizeof(int32_t), std::ios::beg);
  const long long want = static_cast<long long>(kHeaderInts * sizeof(int32_t)) +
                         static_cast<long long>(sections) * static_cast<long long>(*nparams) * 4;
  if (size != want) return fail(LLMK_ERR_INVALID_ARG, std::string("checkpoint: file size does not match the header of ") + path);
  return LLMK_OK;
}

int read_floats(std::ifstream& f, std::vector<float>& v, size_t n, const char* path) {
  v.resize(n);
  if (!f.read(reinterpret_cast<char*>(v.data()), static_cast<std::streamsize>(n * sizeof(float))))
    return fail(LLMK_ERR_INVALID_ARG, std::string("checkpoint: short read in ") + path);
  return LLMK_OK;
}

// Writes header + sections to path.tmp, then renames it over path.
int write_atomically(const char* path, const int32_t* h, const std::vector<const std::vector<float>*>& sections) {
  const std::string tmp = std::string(path) + ".tmp";
  {
    std::ofstream f(tmp, std::ios::binary | std::ios::trunc);
    if (!f.is_open()) return fail(LLMK_ERR_INVALID_ARG, "checkpoint: cannot create " + tmp);
    f.write(reinterpret_cast<const char*>(h), kHeaderInts * sizeof(int32_t));
    for (const auto* s : sections)
      f.write(reinterpret_cast<const char*>(s->data()), static_cast<std::streamsize>(s->size() * sizeof(float)));
    f.flush();
    if (!f) {
      std::remove(tmp.c_str());
      return fail(LLMK_ERR_INVALID_ARG, "checkpoint: write failed for " + tmp);
    }
  }
  if (std::rename(tmp.c_str(), path) != 0) {
    std::remove(tmp.c_str());
    return fail(LLMK_ERR_INVALID_ARG, std::string("checkpoint: cannot rename onto ") + path);
  }
  return LLMK_OK;
}

int model_config(llmk_gpt2* model, llmk_gpt2_config* cfg, size_t* n) {
  if (!model) return fail(LLMK_ERR_INVALID_ARG, "checkpoint: null model");
  LLMK_TRY(llmk_gpt2_get_config(model, cfg));
  *n = llmk_gpt2_parameter_count(model);
  return LLMK_OK;
}

}  // namespace

extern "C" {

int llmk_gpt2_checkpoint_config(const char* path, llmk_gpt2_config* cfg) {
  if (!cfg) return fail(LLMK_ERR_INVALID_ARG, "checkpoint_config: null config");
  std::ifstream f;
  int32_t h[kHeaderInts];
  size_t n;
  return open_checked(f, path, kModelMagic, kModelVersion, 1, h, cfg, &n);
}

int llmk_gpt2_load_checkpoint(llmk_gpt2* model, const char* path) {
  llmk_gpt2_config mc, fc;
  size_t n, fn;
  LLMK_TRY(model_config(model, &mc, &n));
  std::ifstream f;
  int32_t h[kHeaderInts];
  LLMK_TRY(open_checked(f, path, kModelMagic, kModelVersion, 1, h, &fc, &fn));
  if (!same_config(mc, fc)) return fail(LLMK_ERR_INVALID_ARG, std::string("load_checkpoint: configuration differs from the model's in ") + path);
  std::vector<float> p;
  LLMK_TRY(read_floats(f, p, n, path));
  return llmk_gpt2_load_parameters(model, p.data(), n);
}

int llmk_gpt2_save_checkpoint(llmk_gpt2* model, const char* path) {
  llmk_gpt2_config mc;
  size_t n;
  LLMK_TRY(model_config(model, &mc, &n));
  if (!path) return fail(LLMK_ERR_INVALID_ARG, "save_checkpoint: null path");
  std::vector<float> p(n);
  LLMK_TRY(llmk_gpt2_read_parameters(model, p.data(), n));
  int32_t h[kHeaderInts] = {};
  h[0] = kModelMagic;
  h[1] = kModelVersion;
  put_config(h, mc);
  return write_atomically(path, h, {&p});
}

int llmk_gpt2_save_state(llmk_gpt2* model, const char* path, const llmk_train_state* st) {
  llmk_gpt2_config mc;
  size_t n;
  LLMK_TRY(model_config(model, &mc, &n));
  if (!path || !st || st->step < 0 || st->shard_idx < 0 || st->sample_idx < 0)
    return fail(LLMK_ERR_INVALID_ARG, "save_state: bad arguments");
  std::vector<float> p(n), m(n), v(n);
  LLMK_TRY(llmk_gpt2_read_parameters(model, p.data(), n));
  LLMK_TRY(llmk_gpt2_read_optimizer_state(model, m.data(), v.data(), n));
  int32_t h[kHeaderInts] = {};
  h[0] = kStateMagic;
  h[1] = kStateVersion;
  put_config(h, mc);
  h[8] = st->step;
  h[9] = st->world;
  const uint64_t sh = static_cast<uint64_t>(st->shard_idx), sa = static_cast<uint64_t>(st->sample_idx);
  h[10] = static_cast<int32_t>(sh & 0xffffffffu);
  h[11] = static_cast<int32_t>(sh >> 32);
  h[12] = static_cast<int32_t>(sa & 0xffffffffu);
  h[13] = static_cast<int32_t>(sa >> 32);
  return write_atomically(path, h, {&p, &m, &v});
}

int llmk_gpt2_load_state(llmk_gpt2* model, const char* path, llmk_train_state* st) {
  llmk_gpt2_config mc, fc;
  size_t n, fn;
  LLMK_TRY(model_config(model, &mc, &n));
  if (!st) return fail(LLMK_ERR_INVALID_ARG, "load_state: null state");
  std::ifstream f;
  int32_t h[kHeaderInts];
  LLMK_TRY(open_checked(f, path, kStateMagic, kStateVersion, 3, h, &fc, &fn));
  if (!same_config(mc, fc)) return fail(LLMK_ERR_INVALID_ARG, std::string("load_state: configuration differs from the model's in ") + path);
  std::vector<float> p, m, v;
  LLMK_TRY(read_floats(f, p, n, path));
  LLMK_TRY(read_floats(f, m, n, path));
  LLMK_TRY(read_floats(f, v, n, path));
  LLMK_TRY(llmk_gpt2_load_parameters(model, p.data(), n));
  LLMK_TRY(llmk_gpt2_load_optimizer_state(model, m.data(), v.data(), n));
  auto u32 = [](int32_t x) { return static_cast<uint64_t>(static_cast<uint32_t>(x)); };
  st->step = h[8];
  st->world = h[9];
  st->shard_idx = static_cast<long long>(u32(h[10]) | (u32(h[11]) << 32));
  st->sample_idx = static_cast<long long>(u32(h[12]) | (u32(h[13]) << 32));
  return LLMK_OK;
}

}  // extern "C"
