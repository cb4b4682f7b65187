/*
 * qedge_sample.h — C ABI of the B200 token sampler (libqesample.so).
 *
 * This library replaces the sampling step of QEdge's decode loop:
 *   BatchSampler.forward(logits, temperatures, top_ps, *, all_greedy, use_top_p)
 *   (reference: src/compute/sampler.py:25-41), called from
 *   ModelRunner._sample_gpu (src/compute/model_runner.py:77-93) with the
 *   per-row parameters packed by Batch._fill_sampling (src/data/batch.py:149-175).
 *
 * All pointers except `args` itself are device pointers unless stated.
 * Functions never allocate device memory: scratch comes from the caller's
 * workspace, sized by qe_sample_workspace_size().  They return a status
 * code (QE_OK = 0, negative on error) and never abort; the message of the
 * last error on the calling thread is returned by qe_last_error().
 */
#ifndef QEDGE_SAMPLE_H
#define QEDGE_SAMPLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QE_ABI_VERSION 2

/* element type of the logits rows */
enum qe_dtype { QE_DTYPE_F32 = 0, QE_DTYPE_BF16 = 1, QE_DTYPE_F16 = 2 };

/* qe_sample_args.flags */
enum qe_flags {
  QE_FLAG_ALL_GREEDY = 1u, /* BatchSampler.forward(all_greedy=True) (sampler.py:28-29) */
  QE_FLAG_USE_TOP_P = 2u,  /* BatchSampler.forward(use_top_p=True)  (sampler.py:34-38) */
  QE_FLAG_MULTI_KERNEL = 4u /* run the five-launch cross-check path instead of the default
                               single streaming launch (no min_ps, out_kept, out_norm) */
};

/* status codes */
enum qe_status {
  QE_OK = 0,
  QE_ERR_INVALID = -1,     /* bad argument (null pointer, size, alignment) */
  QE_ERR_CUDA = -2,        /* a CUDA call or kernel launch failed */
  QE_ERR_WORKSPACE = -3,   /* workspace missing or smaller than required */
  QE_ERR_UNSUPPORTED = -4  /* a size this build does not handle */
};

/* per-row status bits written to out_status (when non-NULL) */
enum qe_row_status {
  QE_ROW_GREEDY = 1,       /* row sampled as greedy argmax (T <= 1e-5 or all_greedy) */
  QE_ROW_NONFINITE = 2,    /* probabilities not finite; greedy argmax returned */
  QE_ROW_GATHERED = 4,     /* diagnostic: finished from the gathered head of the row */
  QE_ROW_SLOW = 8,         /* diagnostic: finished by the exact (threshold + race) rounds */
  QE_ROW_TIMEOUT = 16      /* reserved: no kernel of this library waits on another CTA or a flag */
};

typedef struct qe_sample_args {
  uint32_t struct_size;        /* sizeof(qe_sample_args) (ABI check) */
  int32_t dtype;               /* enum qe_dtype */
  int64_t batch;               /* B rows */
  int64_t vocab;               /* V ids per row, 1 <= V < 2^24 */
  int64_t ld;                  /* row stride of logits in elements (>= V) */
  const void* logits;          /* [B, ld] logits (sampler.py:25 `logits`) */
  const float* temperatures;   /* [B] (sampler.py:25 `temperatures`; greedy iff <= 1e-5) */
  const float* top_ps;         /* [B] or NULL (sampler.py:26 `top_ps`) */
  const int32_t* top_ks;       /* [B] or NULL; <= 0 or >= V means off (batch.py:154-157) */
  const float* min_ps;         /* [B] or NULL; drop ids with p < min_p * max p (batch.py:60, 158) */
  const float* rep_penalties;  /* [B] or NULL; repetition penalty over the history set */
  const int32_t* history;      /* [B, history_ld] token ids or NULL */
  const int32_t* history_lens; /* [B] valid entries per row, or NULL for all history_ld */
  int64_t history_ld;
  const float* noise;          /* [B, noise_ld] Exp(1) noise (parity mode) or NULL (Philox) */
  int64_t noise_ld;
  uint64_t seed;               /* Philox key of every row ... */
  const uint64_t* seeds;       /* ... or [B] per-row keys (SamplingParams.seed), or NULL */
  uint64_t step;               /* Philox step (decode step) */
  const uint64_t* step_ptr;    /* device step counter; overrides `step` when non-NULL */
  int64_t row_offset;          /* global index of row 0 (keys the Philox stream) */
  uint32_t flags;              /* enum qe_flags */
  uint32_t wait_polls;         /* reserved, ignored: no kernel of this library spins on a wait */
  int64_t* out_ids;            /* [B] sampled token ids (int64, like torch.argmax) */
  float* out_probs;            /* [B, probs_ld] softmax probabilities or NULL */
  int64_t probs_ld;
  int32_t* out_status;         /* [B] enum qe_row_status bits or NULL */
  int64_t* out_kept;           /* debug, [B] or NULL: size of the kept set (0 for greedy and
                                  non-finite rows, V without filters); forces the exact rounds */
  double* out_norm;            /* debug, [B] or NULL: sum_j exp((x_j - max x) / T) */
  void* workspace;             /* device scratch, >= qe_sample_workspace_size() bytes */
  size_t workspace_bytes;
} qe_sample_args;

/* ABI version of the loaded library (QE_ABI_VERSION). */
int qe_abi_version(void);

/* Bytes of device workspace qe_sample needs for a batch of B rows of V ids
 * (enough for either path).  The library never needs it zeroed. */
size_t qe_sample_workspace_size(int64_t batch, int64_t vocab);

/* Sample one token per row on `stream` (a cudaStream_t; NULL = legacy default
 * stream).  Replaces BatchSampler.forward (src/compute/sampler.py:25-41);
 * asynchronous, no host synchronisation, no allocation. */
int qe_sample(const qe_sample_args* args, void* stream);

/* Message of the last error returned on this thread ("" if none). */
const char* qe_last_error(void);

/* Device-side error bits of the last qe_sample call that used `workspace`
 * on the default (streaming) path (4: a race found no candidate, which a row
 * with finite probabilities cannot produce; its id is -1).  Waits for
 * `stream`, then copies one word to the host.  This is the only call of the
 * library that synchronises the host. */
int qe_sample_errors(const void* workspace, void* stream, uint32_t* flags);

/* Bytes of the scratch array built into the library for qe_sample_noalloc. */
#define QE_NOALLOC_SCRATCH_BYTES (32u << 20)

/* qe_sample without a caller workspace (it has no counterpart in the
 * reference).  For callers that cannot allocate device memory: plugins inside
 * a host engine that owns every device allocation, language bindings with no
 * device-memory API.  Same kernels and results as qe_sample; the scratch
 * comes from one QE_NOALLOC_SCRATCH_BYTES array inside the library, which
 * every GPU that uses the library holds until the process exits.
 * `workspace` and `workspace_bytes` in args are ignored.  Calls whose
 * qe_sample_workspace_size(batch, vocab) exceeds the array are rejected with
 * QE_ERR_UNSUPPORTED (at V = 248,320 up to 314 rows fit).  The first call on
 * a device looks up the array's device address; make that first call before
 * any stream capture.  The address is kept for the life of the process: it
 * does not survive cudaDeviceReset or a new primary context on that device.  All calls share the one array: calls that overlap on
 * the GPU (other streams, other host threads) race and must be serialised by
 * the caller.  No part of the array needs to start at zero: every kernel
 * writes the scratch it reads first.  Allocates nothing. */
int qe_sample_noalloc(const qe_sample_args* args, void* stream);

/* ------------------------------------------------------------------------
 * Vocab-sharded sampling (tensor-parallel lm_head).  The reference samples
 * one full [B, V] logits tensor (src/compute/sampler.py:25-41); these calls
 * let each of `nshards` GPUs (1, 2, 4, 8 or 16) keep its own contiguous
 * block of the vocabulary: shard s holds canonical slices
 * [s*16/nshards, (s+1)*16/nshards), i.e. ids
 * [floor(s*V/(8*nshards))*8, floor((s+1)*V/(8*nshards))*8).  In every call
 * `args->vocab` is the full V, `args->logits` (and `noise`) point at the
 * shard's first column with row stride `ld` (`noise_ld`), and the other
 * fields mean what they mean for qe_sample (`workspace` is unused).  V must be
 * <= 262,144.  A step:
 *   1. qe_shard_summarize   -> records [B][16/nshards] on every GPU
 *   2. all-gather records   -> [nshards][B][16/nshards] (e.g. NCCL)
 *   3. qe_shard_merge       -> out_ids for every row that needs no test;
 *                              tests [B] for the rest (identical on every GPU)
 *   4. qe_shard_test        -> partials [B][16/nshards]
 *   5. all-gather partials  -> [nshards][B][16/nshards]
 *   6. qe_shard_decide      -> the remaining out_ids.  A row whose candidates
 *      all fall outside its kept set gets id -1 and status QE_ROW_SLOW; the
 *      caller finishes it exactly (gather that row, call qe_sample).
 * Greedy, small top-k (<= 64) and unfiltered rows are final after step 3.
 * Token ids equal the single-GPU ones under the same noise. */
size_t qe_shard_record_bytes(void);   /* bytes per (row, slice) record */
size_t qe_shard_test_bytes(void);     /* bytes per row of `tests` */
size_t qe_shard_partial_bytes(void);  /* bytes per (row, slice) partial */
int qe_shard_summarize(const qe_sample_args* args, int shard, int nshards, void* records, void* stream);
int qe_shard_merge(const qe_sample_args* args, int nshards, const void* all_records, void* tests, void* stream);
int qe_shard_test(const qe_sample_args* args, int shard, int nshards, const void* tests, void* partials,
                  void* stream);
int qe_shard_decide(const qe_sample_args* args, int nshards, const void* tests, const void* all_partials,
                    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QEDGE_SAMPLE_H */
