// Launchers of the Quest kernels (quest.cu), called by the C ABI after validation.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>

#include "../../include/pbk.h"

namespace pbk {
// Always-visible keys placed before the retrieved pages (the serving path's sink
// positions): n rows of k / v at element strides s_kv (key head) and s_n (row).
struct SinkKeys {
  const __nv_bfloat16* k = nullptr;
  const __nv_bfloat16* v = nullptr;
  int64_t s_kv = 0, s_n = 0;
  int n = 0;
};
int quest_k(const pbk_quest_desc& d);
int quest_splits(const pbk_quest_desc& d, int n_sink);
size_t quest_score_bytes(const pbk_quest_desc& d);
size_t quest_select_floats(const pbk_quest_desc& d);
// Floats of the fixed scratch of pbk_quest_select_noalloc: the largest allowed score count
// plus its segment maxima (rows of at least 1024 pages keep ceil(pages / 32) of them) and
// the tile bound magnitudes (two per 128 pages and key head: at most scores / 32 for rows
// of at least 128 pages).
constexpr size_t kNoAllocFloats = (size_t)PBK_QUEST_NOALLOC_MAX_SCORES + PBK_QUEST_NOALLOC_MAX_SCORES / 32 +
                                  PBK_QUEST_NOALLOC_MAX_SCORES / 1024 + PBK_QUEST_NOALLOC_MAX_SCORES / 32;
size_t quest_partial_bytes(const pbk_quest_desc& d, int n_sink);
cudaError_t launch_quest_select(const pbk_quest_desc& d, float* scratch, cudaStream_t st);
cudaError_t launch_quest_select_parts(const pbk_quest_desc& d, float* scratch, int parts, cudaStream_t st);
bool quest_score_tc_supported(const pbk_quest_desc& d);
// Tiles of 128 pages per key head and values per tile in the score kernel's tile_abs output.
int quest_score_tc_tiles(const pbk_quest_desc& d);
int quest_score_tc_abs_slots();
cudaError_t launch_quest_score_tc(const pbk_quest_desc& d, float* scores, float* segmax, int nseg, float* tile_abs,
                                  cudaStream_t st);
cudaError_t launch_quest_select_noalloc(const pbk_quest_desc& d, cudaStream_t st);
// parts (bit mask): 1 the retrieved splits, 2 the window splits, 4 the combine (all: 7).
cudaError_t launch_quest_attend(const pbk_quest_desc& d, float* part, const SinkKeys& sk, int parts, cudaStream_t st);
// Tensor-core split attention (quest_attend_mma.cu): up to 16 query rows per key head.
bool quest_attend_mma_supported(const pbk_quest_desc& d);
// It picks its own split length (>= the SIMT kernel's, so the workspace sized by
// quest_partial_bytes holds its partials) and returns the splits per (query, key head).
// parts: 1 the retrieved splits, 2 the window splits (both: 3).
cudaError_t launch_quest_attend_mma(const pbk_quest_desc& d, int k, int tail, float* part, const SinkKeys& sk,
                                    int parts, int* splits, cudaStream_t st);
// Exact rescoring of c candidate pages [nq, kv, c] (ascending) and selection of the best
// k = min(budget, c) into desc.pages, ascending; `exact` holds nq * kv * c floats.
cudaError_t launch_quest_rerank(const pbk_quest_desc& d, const int32_t* cand, int c, float* exact, cudaStream_t st);
cudaError_t launch_quest_gather(const pbk_quest_desc& d, int sel, void* ok, void* ov, cudaStream_t st);
// Two-level / hole-masked selection (pbk_quest_select_levels): workspace bytes and launch.
size_t quest_levels_bytes(const pbk_quest_desc& d, const pbk_quest_levels& lv);
cudaError_t launch_quest_select_levels(const pbk_quest_desc& d, const pbk_quest_levels& lv, uint8_t* ws,
                                       cudaStream_t st);
cudaError_t launch_quest_superbounds(const void* kmax, const void* kmin, int kv, int n_blk, int dim, int sblk,
                                     int64_t bs_kv, int64_t bs_p, void* smax, void* smin, int64_t ss_kv, int64_t ss_p,
                                     int first_sb, int end_sb, cudaStream_t st);
cudaError_t launch_quest_rope_gather(const pbk_rope_gather_desc& d, cudaStream_t st);
cudaError_t launch_quest_archive_write(const pbk_archive_write_desc& d, cudaStream_t st);
cudaError_t launch_quest_supermeans(const void* bmean, int kv, int n_blk, int dim, int sblk, int64_t bs_kv,
                                    int64_t bs_p, void* smean, int64_t ss_kv, int64_t ss_p, int first_sb, int end_sb,
                                    cudaStream_t st);
cudaError_t launch_quest_bounds(const void* keys, int kv, int n, int dim, int page, int64_t ks_kv, int64_t ks_n,
                                void* kmax, void* kmin, int64_t bs_kv, int64_t bs_p, int first_page, cudaStream_t st);
}  // namespace pbk
