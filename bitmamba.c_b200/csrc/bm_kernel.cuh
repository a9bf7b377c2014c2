// Internal interface between the C ABI (bm_sampler.cu) and the sampling
// kernel (bm_kernel.cu).  Not part of the public ABI.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "bm_sampler.h"

namespace bmk {

constexpr int NT = 512;       // threads per CTA (one CTA per SM)
constexpr int NW = NT / 32;   // warps per CTA
constexpr int HB = 128;       // reference histogram buckets (src/model.c:132)
constexpr int NB = 2048;      // full-vocabulary path: logit buckets
constexpr int WCAP = 1024;    // full-vocabulary path: window list capacity
constexpr int KCAP = 2048;    // top_k path: candidate list capacity
constexpr int NCHUNK = 8;     // bulk-copy chunks (one mbarrier each) per row
constexpr int SCRATCH = 22528;

struct Params {
    const float *logits;
    int64_t ld;
    int B, V;
    const int32_t *hist;
    const int64_t *hist_off;
    const bm_knobs_t *knobs;
    int64_t knob_stride;
    const float *uniform;
    int32_t *out_id;
    float *out_prob;
    bm_row_stats_t *stats;
    int *err;    // device error word: bit 0 = bounded wait expired, bit 1 = an
                 // exact select did not converge
    int *sched;  // row schedule: [0] rows claimed past the first grid, [1] CTAs
                 // finished; both zero between launches
    int mark_failed_rows = 0;  // nonzero: a row whose bounded wait expired or
                               // whose exact select did not converge gets id
                               // -1, and the last CTA clears the error word
    const int *dB = nullptr;   // optional: the row count, read at launch from
                               // this device word (at most B)
    const int32_t *row_map = nullptr;  // optional: launch row i is row
                                       // row_map[i] of every per-row array,
                                       // the logits included
};

// The merge kernel of the fused lm_head + sampler: per row, the per-tile
// lists of the GEMM's summary epilogue (tiles x ks entries, (bits(value) <<
// 32) | id) finish the greedy argmax or the top_k path; rows they cannot
// decide, and rows of the full-vocabulary path, are appended to the fallback
// lists (fb = [count, rows...]: to be sampled from logits; nl = [count,
// rows...]: their logits still to be computed).
struct SumParams {
    const uint64_t *summ;
    int tiles, ks;
    int B, V;
    const bm_knobs_t *knobs;
    int64_t knob_stride;
    const float *uniform;
    int32_t *out_id;
    float *out_prob;
    bm_row_stats_t *stats;
    int *fb;
    int *nl;
    int *err;
};
// The merge kernel's rows are independent and its serial phases short of
// work, so several CTAs share an SM (their phases overlap).
constexpr int MERGE_CTAS_PER_SM = 4;
cudaError_t launch_summary(const SumParams &p, int grid, cudaStream_t s);
cudaError_t prepare_summary(int V, int tiles, int ks);

// Dynamic shared memory the kernel needs for vocabulary V.
size_t smem_bytes(int V);
// Largest V whose row buffer fits in `smem_limit` bytes of shared memory.
int max_vocab(size_t smem_limit);
// Launch on `grid` CTAs (one per SM is the intended shape).
cudaError_t launch(const Params &p, int grid, cudaStream_t s);
// One-time per-device attribute setup (dynamic shared memory opt-in).
cudaError_t prepare(int V);
// The calling thread's current device's copy of a file-scope device array of
// NOALLOC_WORDS ints (256-byte aligned): word 0 error bits, words 1-2 the row
// schedule counters (zero at module load, returned to zero by every launch).
constexpr int NOALLOC_WORDS = 64;
cudaError_t noalloc_scratch(int **out);

}  // namespace bmk
