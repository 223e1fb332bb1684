// llmk_dataloader.hpp — the reference's DataLoader class over the llmk C ABI.
//
// Header-only adapter: a maintainer includes this instead of the reference's
// utils/dataloader.h and the training programs compile unchanged. Same
// constructor arguments (utils/dataloader.h:62-66), NextBatch overloads
// (utils/dataloader.h:79-89), Resume / Reset and the public num_tokens
// member. Where the reference prints and exit()s on a bad shard
// (utils/dataloader.cpp:36-39,73-106) or throws std::invalid_argument on a
// batch of the wrong size (utils/dataloader.cpp:122-128), this class throws
// std::invalid_argument with the library's message.
#pragma once

#include <cstddef>
#include <filesystem>
#include <stdexcept>
#include <string>
#include <vector>

#include "llmk_data.h"

class DataLoader {
 public:
  DataLoader() = delete;
  DataLoader(const DataLoader&) = delete;
  DataLoader& operator=(const DataLoader&) = delete;

  explicit DataLoader(const std::filesystem::path& shard_dir, size_t B, size_t T, unsigned int process_rank,
                      unsigned int num_processes, bool should_shuffle)
      : B_(B), T_(T), in_(B * T), tg_(B * T) {
    check(llmk_loader_create(&h_, shard_dir.string().c_str(), static_cast<int>(B), static_cast<int>(T),
                             static_cast<int>(process_rank), static_cast<int>(num_processes), should_shuffle ? 1 : 0));
    num_tokens = static_cast<size_t>(llmk_loader_num_tokens(h_));
  }
  ~DataLoader() { llmk_loader_destroy(h_); }

  template <class InputIterator, class OutputIterator>
  void NextBatch(InputIterator input, OutputIterator target) {
    check(llmk_loader_next(h_, in_.data(), tg_.data()));
    for (size_t i = 0; i < B_ * T_; ++i, ++input, ++target) {
      *input = in_[i];
      *target = tg_[i];
    }
  }

  void NextBatch(std::vector<int>& inputs, std::vector<int>& targets) {
    if (inputs.size() != B_ * T_) throw std::invalid_argument("inputs size mismatch");
    if (targets.size() != B_ * T_) throw std::invalid_argument("outputs size mismatch");
    check(llmk_loader_next(h_, inputs.data(), targets.data()));
  }

  void Resume(size_t shard_idx, size_t sample_idx) { check(llmk_loader_resume(h_, shard_idx, sample_idx)); }
  void Reset() { check(llmk_loader_reset(h_)); }

  // Not in the reference: the position Resume takes, for checkpointing.
  void Position(size_t* shard_idx, size_t* sample_idx) const { check(llmk_loader_position(h_, shard_idx, sample_idx)); }

  size_t num_tokens = 0;

 private:
  static void check(int rc) {
    if (rc != LLMK_OK) throw std::invalid_argument(std::string("DataLoader: ") + llmk_last_error());
  }
  llmk_loader* h_ = nullptr;
  size_t B_, T_;
  std::vector<int> in_, tg_;
};
