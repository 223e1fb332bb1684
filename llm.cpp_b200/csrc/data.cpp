// Token-shard data loader (host side): see include/llmk_data.h for the file
// format, the batch order and the reference functions each entry replaces.
//
// The shuffle has to draw the same permutations as the reference
// (utils/rand.h: Fisher-Yates from the back with std::uniform_int_distribution
// on std::mt19937) for a run to see the reference's batch sequence, so it uses
// the same standard-library engine and distribution in the same order.
#include <cstdint>
#include <cstdio>
#include <filesystem>
#include <fstream>
#include <numeric>
#include <random>
#include <string>
#include <vector>

#include "llmk_data.h"
#include "runtime.h"

namespace fs = std::filesystem;
using llmk::fail;

struct llmk_loader {
  static constexpr int kHeaderInts = 256;
  static constexpr int kMagic = 20240520;
  size_t B = 0, T = 0;
  unsigned rank = 0, world = 1;
  bool shuffle = false;
  std::vector<fs::path> shards;
  std::vector<int> shard_order;   // shuffled shard indices
  std::vector<int> sample_order;  // shuffled sample indices of the open shard
  std::mt19937 rng;
  std::ifstream file;
  size_t shard_samples = 0;  // samples of the open shard for this rank
  size_t shard_idx = 0, sample_idx = 0;
  long long num_tokens = 0;
  std::vector<uint16_t> buf;
};

namespace {

void permute(std::vector<int>& v, std::mt19937& rng) {
  for (int i = static_cast<int>(v.size()) - 1; i > 0; --i) {
    std::uniform_int_distribution<int> pick{0, i};
    const int j = pick(rng);
    std::swap(v[i], v[j]);
  }
}

// Opens shard `i` (through the shuffled order when shuffling) and validates it;
// *ntok = its token count.
int open_shard(llmk_loader* l, size_t i, long long* ntok) {
  const size_t k = l->shuffle ? static_cast<size_t>(l->shard_order[i]) : i;
  const fs::path& p = l->shards[k];
  if (l->file.is_open()) l->file.close();
  l->file.clear();
  l->file.open(p, std::ios::binary);
  if (!l->file.is_open()) return fail(LLMK_ERR_INVALID_ARG, "loader: cannot open " + p.string());
  int32_t header[llmk_loader::kHeaderInts];
  if (!l->file.read(reinterpret_cast<char*>(header), sizeof(header)))
    return fail(LLMK_ERR_INVALID_ARG, "loader: cannot read the header of " + p.string());
  if (header[0] != llmk_loader::kMagic) return fail(LLMK_ERR_INVALID_ARG, "loader: bad magic in " + p.string());
  if (header[1] != 1) return fail(LLMK_ERR_INVALID_ARG, "loader: bad version in " + p.string());
  const long long n = header[2];
  if (n <= 0) return fail(LLMK_ERR_INVALID_ARG, "loader: no tokens in " + p.string());
  l->file.seekg(0, std::ios::end);
  const long long size = static_cast<long long>(l->file.tellg());
  l->file.seekg(0, std::ios::beg);
  if (size != static_cast<long long>(sizeof(header)) + n * 2)
    return fail(LLMK_ERR_INVALID_ARG, "loader: file size does not match the token count of " + p.string());
  // B*T+1 tokens are read per sample while samples advance by B*T
  l->shard_samples = static_cast<size_t>((n * 2 - 2) / static_cast<long long>(l->world * l->B * l->T * 2));
  *ntok = n;
  return LLMK_OK;
}

void order_samples(llmk_loader* l) {
  l->sample_order.assign(l->shard_samples, 0);
  std::iota(l->sample_order.begin(), l->sample_order.end(), 0);
  permute(l->sample_order, l->rng);
}

int reset(llmk_loader* l) {
  l->shard_idx = 0;
  l->sample_idx = 0;
  if (l->shuffle) permute(l->shard_order, l->rng);
  long long n;
  LLMK_TRY(open_shard(l, 0, &n));
  if (l->shuffle) order_samples(l);
  return LLMK_OK;
}

int advance(llmk_loader* l) {
  if (l->shard_idx + 1 == l->shards.size()) return reset(l);
  l->shard_idx = (l->shard_idx + 1) % l->shards.size();
  l->sample_idx = 0;
  long long n;
  LLMK_TRY(open_shard(l, l->shard_idx, &n));
  if (l->shuffle) order_samples(l);
  return LLMK_OK;
}

}  // namespace

extern "C" {

int llmk_loader_create(llmk_loader** out, const char* path, int B, int T, int rank, int world, int shuffle) {
  if (!out || !path || B <= 0 || T <= 0 || world <= 0 || rank < 0 || rank >= world)
    return fail(LLMK_ERR_INVALID_ARG, "loader_create: bad arguments");
  *out = nullptr;
  auto* l = new llmk_loader();
  l->B = static_cast<size_t>(B);
  l->T = static_cast<size_t>(T);
  l->rank = static_cast<unsigned>(rank);
  l->world = static_cast<unsigned>(world);
  l->shuffle = shuffle != 0;
  std::error_code ec;
  const fs::path p{path};
  if (fs::is_regular_file(p, ec)) {
    l->shards.push_back(p);
  } else if (fs::is_directory(p, ec)) {
    for (const auto& e : fs::directory_iterator{p, ec})
      if (e.is_regular_file()) l->shards.push_back(e.path());
  }
  if (l->shards.empty()) {
    delete l;
    return fail(LLMK_ERR_INVALID_ARG, std::string("loader_create: no shard file at ") + path);
  }
  if (l->shuffle) {
    l->rng.seed(42u + static_cast<unsigned>(world));
    l->shard_order.assign(l->shards.size(), 0);
    std::iota(l->shard_order.begin(), l->shard_order.end(), 0);
  }
  const long long need = static_cast<long long>(world) * B * T + 1;
  for (size_t i = 0; i < l->shards.size(); ++i) {
    long long n = 0;
    int rc = open_shard(l, i, &n);
    if (rc == LLMK_OK && n < need) rc = fail(LLMK_ERR_INVALID_ARG, "loader_create: a shard holds fewer than world*B*T+1 tokens");
    if (rc != LLMK_OK) {
      delete l;
      return rc;
    }
    l->num_tokens += n;
  }
  l->buf.resize(static_cast<size_t>(B) * T + 1);
  const int rc = reset(l);
  if (rc != LLMK_OK) {
    delete l;
    return rc;
  }
  *out = l;
  return LLMK_OK;
}

int llmk_loader_destroy(llmk_loader* l) {
  delete l;
  return LLMK_OK;
}

int llmk_loader_next(llmk_loader* l, int* inputs, int* targets) {
  if (!l || !inputs || !targets) return fail(LLMK_ERR_INVALID_ARG, "loader_next: null argument");
  if (l->sample_idx >= l->shard_samples) LLMK_TRY(advance(l));
  // After a Resume into a shard with more samples than the last shuffled
  // order holds, the reference would index past that order; refuse instead.
  if (l->shuffle && l->sample_idx >= l->sample_order.size())
    return fail(LLMK_ERR_INVALID_ARG, "loader_next: resumed position is outside the shuffled sample order");
  const size_t idx = l->shuffle ? static_cast<size_t>(l->sample_order[l->sample_idx]) : l->sample_idx;
  const size_t bt = l->B * l->T;
  const long long off = static_cast<long long>(llmk_loader::kHeaderInts) * 4 +
                        static_cast<long long>(idx) * l->world * bt * 2 + static_cast<long long>(l->rank) * bt * 2;
  l->file.clear();
  l->file.seekg(off, std::ios::beg);
  if (!l->file.read(reinterpret_cast<char*>(l->buf.data()), static_cast<std::streamsize>(l->buf.size() * 2)))
    return fail(LLMK_ERR_INVALID_ARG, "loader_next: short read");
  for (size_t i = 0; i < bt; ++i) {
    inputs[i] = static_cast<int>(l->buf[i]);
    targets[i] = static_cast<int>(l->buf[i + 1]);
  }
  ++l->sample_idx;
  return LLMK_OK;
}

int llmk_loader_reset(llmk_loader* l) {
  if (!l) return fail(LLMK_ERR_INVALID_ARG, "loader_reset");
  return reset(l);
}

int llmk_loader_resume(llmk_loader* l, size_t shard_idx, size_t sample_idx) {
  if (!l || shard_idx >= l->shards.size()) return fail(LLMK_ERR_INVALID_ARG, "loader_resume: bad position");
  l->shard_idx = shard_idx;
  l->sample_idx = sample_idx;
  long long n;
  return open_shard(l, shard_idx, &n);
}

int llmk_loader_position(const llmk_loader* l, size_t* shard_idx, size_t* sample_idx) {
  if (!l) return fail(LLMK_ERR_INVALID_ARG, "loader_position");
  if (shard_idx) *shard_idx = l->shard_idx;
  if (sample_idx) *sample_idx = l->sample_idx;
  return LLMK_OK;
}

long long llmk_loader_num_tokens(const llmk_loader* l) { return l ? l->num_tokens : -1; }

}  // extern "C"
