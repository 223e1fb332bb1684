/* llmk_data.h — token-shard data loader (host side), C ABI.
 *
 * The B200 counterpart of the reference's DataLoader (utils/dataloader.h,
 * utils/dataloader.cpp), with the same file format and batch order:
 *
 *  - a shard is a file of 256 int32 header words (magic 20240520, version 1,
 *    token count) followed by that many uint16 tokens
 *    (utils/dataloader.cpp:84-115);
 *  - `path` is one shard or a directory whose regular files are the shards,
 *    in directory-iteration order (utils/dataloader.cpp:26-40);
 *  - rank r of `world` reads B*T+1 tokens at sample i from byte
 *    1024 + i*world*B*T*2 + r*B*T*2 of its shard: inputs are the first B*T
 *    tokens, targets the B*T tokens after the first (utils/dataloader.cpp:147-156);
 *  - with shuffling, shard order and the sample order inside each shard are
 *    permuted by Fisher-Yates with std::mt19937 seeded 42 + world and
 *    std::uniform_int_distribution, drawing in the reference's sequence
 *    (utils/rand.h, utils/dataloader.cpp:42-48,189-216);
 *  - past the last sample of a shard the next shard is opened; past the last
 *    shard the loader resets (re-permuting the shards).
 *
 * Errors are status codes (llmk_status.h) with llmk_last_error() text
 * (llmk.h); the reference prints and exit()s or asserts. */
#ifndef LLMK_DATA_H_
#define LLMK_DATA_H_

#include <stddef.h>

#include "llmk.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct llmk_loader llmk_loader;

/* Replaces DataLoader::DataLoader(shard_dir, B, T, process_rank,
 * num_processes, should_shuffle), utils/dataloader.cpp:15-60. Fails when a
 * shard has a bad header or size, or fewer than world*B*T+1 tokens. */
int llmk_loader_create(llmk_loader** out, const char* path, int B, int T, int rank, int world, int shuffle);
int llmk_loader_destroy(llmk_loader* loader);
/* Replaces DataLoader::NextBatch (utils/dataloader.h:79-87): inputs and
 * targets are host arrays of B*T ints. */
int llmk_loader_next(llmk_loader* loader, int* inputs, int* targets);
/* DataLoader::Reset / Resume (utils/dataloader.cpp:176-198). */
int llmk_loader_reset(llmk_loader* loader);
int llmk_loader_resume(llmk_loader* loader, size_t shard_idx, size_t sample_idx);
/* Current position (the arguments Resume takes) and the total token count of
 * all shards (DataLoader::num_tokens). */
int llmk_loader_position(const llmk_loader* loader, size_t* shard_idx, size_t* sample_idx);
long long llmk_loader_num_tokens(const llmk_loader* loader);

#ifdef __cplusplus
}
#endif

#endif /* LLMK_DATA_H_ */
