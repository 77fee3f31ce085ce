/*
 * mssample.h -- C ABI of the B200 token-sampling library (libmssample.so).
 *
 * Drop-in boundary for miniserve's sampling hot path.  Each entry point
 * replaces one reference interface, cited below by file:line of the
 * miniserve project:
 *
 *   ms_sample            Sampler.sample (miniserve/sampler.py:23-68), batched:
 *                        one token per row of a [B, V] logits matrix, with
 *                        per-row temperature / top_k / top_p and a
 *                        caller-supplied uniform per row (the value
 *                        random.Random(seed).random() the reference draws at
 *                        miniserve/sampler.py:32,62).  With a mask it also
 *                        applies the logits-processor hook's -inf convention
 *                        (miniserve/model_runner.py:214-216) before sampling.
 *                        Serves the sample_fn(out, plan) -> List[int] seam of
 *                        OverlapEngine (miniserve/overlap.py:109-112).
 *
 * Conventions
 *   - Every pointer argument is a DEVICE pointer owned by the caller.
 *   - Launches are asynchronous on `stream`; nothing is synchronised.
 *   - Return value: MS_OK, or a negative MS_E_* for argument or launch errors
 *     detected on the host before/at launch.
 *   - Per-row conditions are reported in row_status (MS_ROW_* bits); a row
 *     with a non-zero status other than MS_ROW_NONFINITE gets token -1.
 *   - No global mutable state: calls from several host threads on different
 *     streams are safe.
 */
#ifndef MSSAMPLE_H
#define MSSAMPLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *ms_stream_t; /* == cudaStream_t */

enum {
  MS_OK = 0,
  MS_E_INVALID = -1,     /* null pointer, B < 0, V < 1, ld < V, V >= 2^31 ... */
  MS_E_DTYPE = -2,       /* dtype not MS_DTYPE_F32 / MS_DTYPE_BF16 */
  MS_E_CUDA = -3,        /* a CUDA call failed (see ms_last_cuda_error) */
  MS_E_UNSUPPORTED = -4, /* valid request outside what this build handles */
  MS_E_TOO_LARGE = -5    /* a size beyond the fixed device array of
                            ms_build_json_mask_noalloc (V > 262144) */
};

enum { MS_DTYPE_F32 = 0, MS_DTYPE_BF16 = 1 };

/* row_status bits */
enum {
  MS_ROW_OK = 0,
  MS_ROW_ALL_MASKED = 1,      /* temperature > 0 and every logit is -inf/masked:
                                 the reference raises ZeroDivisionError
                                 (miniserve/sampler.py:46-47) */
  MS_ROW_BAD_TEMPERATURE = 2, /* temperature < 0, NaN or infinite */
  MS_ROW_NONFINITE = 4,       /* a NaN or +inf logit was present; NaN is read
                                 as -inf (the reference's result is arbitrary) */
  MS_ROW_UNSUPPORTED = 8,     /* vocab-sharded calls only: the row needs the
                                 full vocabulary (top_k off or above kmax,
                                 a tie block past the candidate buffer, a
                                 non-finite logit); token -1 */
  MS_ROW_PEER_TIMEOUT = 16    /* fused peer exchange only: a rank's record
                                 of the row had not arrived when
                                 ms_exchange_merge gave up waiting; token -1 */
};

/*
 * Sample one token per row.
 *
 *   logits       [B, ld] row-major, fp32 (dtype 0) or bf16 (dtype 1); the
 *                first V entries of each row are the vocabulary.
 *   temperature  [B] f64; 0 selects greedy argmax (first maximal index).
 *   top_k        [B] i32; <= 0 or >= V disables (miniserve/sampler.py:37).
 *   top_p        [B] f64; >= 1 (or NaN) disables (miniserve/sampler.py:49).
 *   uniforms     [B] f64 in [0, 1).
 *   mask         optional [B, mask_ld] u32 bitmask, bit (i & 31) of word
 *                (i >> 5) set = token i allowed; NULL = all allowed.
 *   tokens       [B] i64 out; probs [B] f32 out (final renormalised
 *                probability of the returned token, 1 for greedy);
 *   row_status   [B] i32 out.
 */
int ms_sample(const void *logits, int dtype, int64_t B, int64_t V, int64_t ld,
              const double *temperature, const int32_t *top_k, const double *top_p,
              const double *uniforms, const uint32_t *mask, int64_t mask_ld, int64_t *tokens,
              float *probs, int32_t *row_status, ms_stream_t stream);

/*
 * Same contract and results as ms_sample, always through the multi-pass
 * kernel that re-reads each row from global memory (one CTA per row) instead
 * of the streaming single-read path.  It has no vocabulary-size limit
 * and serves as the cross-check of the fast path.  Same reference interface
 * as ms_sample (miniserve/sampler.py:23-68).
 */
int ms_sample_generic(const void *logits, int dtype, int64_t B, int64_t V, int64_t ld,
                      const double *temperature, const int32_t *top_k, const double *top_p,
                      const double *uniforms, const uint32_t *mask, int64_t mask_ld,
                      int64_t *tokens, float *probs, int32_t *row_status, ms_stream_t stream);

/*
 * Vocab-sharded sampling.  Rank r of N holds the contiguous slice
 * [v0, v0 + Vloc) of a V-token vocabulary (as a tensor-parallel LM head
 * produces it; slices in rank order).  The global top-k is contained in the
 * union of the slices' top-k, so a fixed-size candidate record per row and
 * rank is all that crosses the interconnect:
 *
 *   1. every rank: ms_shard_candidates on its slice -> records [B][rec_words]
 *   2. the caller all-gathers the records of all ranks, rank-major:
 *      [nranks][B][rec_words] (e.g. ncclAllGather)
 *   3. every rank: ms_shard_merge -> the same tokens on every rank
 *
 * Record of one row (32-bit words, rec_words = 4 + 2*kmax): [0] candidate
 * count m <= kmax, [1] MS_ROW_* bits, [2, 2+kmax) order keys of the slice's
 * top-m values (value descending, index ascending), [2+kmax, 2+2*kmax) their
 * global token ids, [2+2*kmax, 4+2*kmax) a float64 (low word first): for rows
 * without top-k, the slice's sum of exp((v - m) / T) over its finite logits,
 * m the slice maximum (0 otherwise).  Greedy rows (temperature 0 or top_k 1)
 * and top-k rows (2 <= top_k <= kmax) are exact.  Top-p rows without top-k
 * (kmax >= 2 < Vloc) are exact when the nucleus lies among the candidates:
 * its crossing value above the kmax-th largest value of every slice whose
 * record is full.  Rows the scheme cannot sample exactly (top_k above kmax,
 * top_k >= Vloc, top_p >= 1 without top-k, a nucleus reaching past the
 * candidates, tie blocks beyond the candidate buffer, non-finite logits)
 * come back with MS_ROW_UNSUPPORTED or MS_ROW_NONFINITE and token -1; the
 * caller samples those rows from their full vocabulary (ms_sample on the
 * gathered row).  Same reference semantics as ms_sample
 * (miniserve/sampler.py:23-68).
 *
 * kmax: 1..256, the same on every rank.  mask: optional bitmask of the slice
 * ([B, mask_ld] u32, bit i = local token i).
 */
int ms_shard_candidates(const void *logits, int dtype, int64_t B, int64_t Vloc, int64_t ld, int64_t v0,
                        int64_t V, const double *temperature, const int32_t *top_k, const uint32_t *mask,
                        int64_t mask_ld, int32_t kmax, uint32_t *records, ms_stream_t stream);

/* 32-bit words of one row's record for a given kmax (4 + 2*kmax). */
int64_t ms_shard_record_words(int32_t kmax);

/*
 * Merge the all-gathered records ([nranks][B][rec_words]) into tokens,
 * probabilities and statuses (same outputs as ms_sample).  nranks * kmax must
 * be <= 2048.
 */
int ms_shard_merge(const uint32_t *records, int32_t nranks, int64_t B, int32_t kmax, int64_t V,
                   const double *temperature, const int32_t *top_k, const double *top_p,
                   const double *uniforms, int64_t *tokens, float *probs, int32_t *row_status,
                   ms_stream_t stream);

/*
 * Fused peer exchange: steps 1-3 above without a collective call.  Each rank
 * owns an exchange buffer (ms_exchange_words words, zeroed, 16-byte aligned)
 * that every other rank has mapped (ms_ipc_handle / ms_ipc_open); peers:
 * device array [nranks] of the buffers' addresses as seen from this rank
 * (peers[rank] = its own).  Per call, every rank, same arguments except the
 * slice and rank:
 *
 *   1. ms_shard_exchange: the slice's records (as ms_shard_candidates) are
 *      stored into every other rank's buffer over NVLink as each row
 *      finishes, every word tagged with the call's epoch in one 8-byte
 *      store (no fence, no wait).
 *   2. ms_exchange_merge: row by row, waits (at most timeout_ns; a stalled
 *      batch up to about twice that) until every other rank's words of the
 *      row carry the epoch; row r is then merged (as ms_shard_merge does) on
 *      rank r mod nranks, which stores the result into every rank's buffer,
 *      tagged the same way (with one rank: straight into the outputs).
 *   3. ms_exchange_results: waits (at most timeout_ns) for every row's
 *      result and writes tokens, probs and statuses (nothing to do with one
 *      rank).  A row with a word or result missing: token -1,
 *      MS_ROW_PEER_TIMEOUT.
 *
 * epoch: the call's number, 1, 2, ... in order on every rank (with a fresh
 * buffer; it may wrap to 1 after an even number).  Bcap / kmax_cap: the
 * buffer's capacity (B <= Bcap, kmax <= kmax_cap, the same on every rank).
 * The call's records stay readable in every buffer, at word
 * ms_exchange_records_offset, in the all-gather layout
 * [nranks][B][rec_words] (the distributed nucleus reads them) until the call
 * after next starts.  Rows flagged MS_ROW_UNSUPPORTED / MS_ROW_NONFINITE take
 * the same paths as after ms_shard_merge.  nranks * kmax <= 2048, nranks <=
 * 256, B <= 2^20.  Replaces the all-gather of the records (no counterpart in
 * the reference, which samples on one device: miniserve/sampler.py:23-68).
 */
int64_t ms_exchange_words(int64_t Bcap, int32_t nranks, int32_t kmax_cap);
int64_t ms_exchange_records_offset(int64_t Bcap, int32_t nranks, int32_t kmax_cap, uint32_t epoch);
int ms_shard_exchange(const void *logits, int dtype, int64_t B, int64_t Vloc, int64_t ld, int64_t v0, int64_t V,
                      const double *temperature, const int32_t *top_k, const double *top_p, const double *uniforms,
                      const uint32_t *mask, int64_t mask_ld, int32_t kmax, uint32_t *xbuf, uint32_t *const *peers,
                      int32_t rank, int32_t nranks, int64_t Bcap, int32_t kmax_cap, uint32_t epoch,
                      ms_stream_t stream);
int ms_exchange_merge(uint32_t *xbuf, uint32_t *const *peers, int32_t rank, int32_t nranks, int64_t B,
                      int64_t Bcap, int32_t kmax,
                      int32_t kmax_cap, int64_t V, const double *temperature, const int32_t *top_k,
                      const double *top_p, const double *uniforms, uint32_t epoch, int64_t timeout_ns,
                      int64_t *tokens, float *probs, int32_t *row_status, ms_stream_t stream);
int ms_exchange_results(const uint32_t *xbuf, int32_t nranks, int64_t B, int64_t Bcap, int32_t kmax_cap,
                        uint32_t epoch, int64_t timeout_ns, int64_t *tokens, float *probs, int32_t *row_status,
                        ms_stream_t stream);

/*
 * Device memory for an exchange buffer and its CUDA IPC mapping into the
 * other ranks' processes (legacy CUDA IPC: no multicast object is made).
 * ms_device_alloc zeroes the block and synchronizes the device.  handle: 64
 * bytes (cudaIpcMemHandle_t), exchanged by the caller (e.g. an all-gather of
 * bytes).  ms_ipc_open maps a peer's block with peer access enabled.
 */
int ms_device_alloc(int64_t bytes, void **ptr);
int ms_device_free(void *ptr);
int ms_ipc_handle(void *ptr, unsigned char *handle);
int ms_ipc_open(const unsigned char *handle, void **ptr);
int ms_ipc_close(void *ptr);

/*
 * The distributed nucleus: vocab-sharded rows without top-k that
 * ms_shard_merge flags MS_ROW_UNSUPPORTED (a nucleus wider than the
 * candidates, or top_p >= 1), sampled without gathering their logits
 * (miniserve/sampler.py:35-68 with top_k off).  rows: [F] the batch rows to
 * finish; records: the all-gathered candidate records of the merge
 * ([nranks][B][rec_words], kmax >= 2), which give each row's maximum.  Every
 * rank, in this order:
 *
 *   1. ms_nucleus_hist on its slice -> hist [F][hist_words] u32 (fixed-point
 *      histogram of the row's weights over (max - logit) / T, scaled from V
 *      so that the sum over all ranks stays below 2^31)
 *   2. the caller all-reduces hist (sum, as int32)
 *   3. ms_nucleus_bracket -> bracket [F][2] i32 (the bins holding the top-p
 *      crossing; identical on every rank)
 *   4. ms_nucleus_classify on its slice -> entries [F][record_words] u32 (the
 *      slice's mass above the bracket and in all, the bracket's values) and
 *      segments [F][ms_nucleus_segments()] f64 (the mass above the bracket
 *      of each index-order segment of the slice; stays on the rank)
 *   5. the caller all-gathers entries rank-major: [nranks][F][record_words]
 *   6. ms_nucleus_cut -> cut [F][cut_words] u32 (the crossing entry, the
 *      rank whose slice holds the draw's target; identical on every rank).
 *      bounds: [nranks + 1] i64, the slices' first global ids and V.
 *   7. ms_nucleus_draw on its slice (with the all-gathered entries and its
 *      own segments) -> out [F][2] i64: (token, float bits of its
 *      probability) on the owning rank, (-1, 0) elsewhere
 *   8. the caller all-reduces out (max): every rank has each row's token.
 *
 * A row whose cut record's status word ([3]) is nonzero (its bracket held
 * more than 2048 of a slice's values, or the histogram missed the crossing)
 * comes back with token -1 from step 7 and is left to the full-row path.
 * Vloc <= 2^20, V < 2^27, nranks <= 256.
 */
int64_t ms_nucleus_hist_words(void);
int64_t ms_nucleus_record_words(void);
int64_t ms_nucleus_cut_words(void);
int64_t ms_nucleus_segments(void);
int ms_nucleus_hist(const void *logits, int dtype, int64_t Vloc, int64_t ld, const uint32_t *mask, int64_t mask_ld,
                    const int32_t *rows, int64_t F, int64_t B, int64_t V, const uint32_t *records, int32_t nranks,
                    int32_t kmax, const double *temperature, const double *top_p, uint32_t *hist,
                    ms_stream_t stream);
int ms_nucleus_bracket(const uint32_t *hist, const int32_t *rows, int64_t F, int64_t V, const double *top_p,
                       int32_t *bracket, ms_stream_t stream);
int ms_nucleus_classify(const void *logits, int dtype, int64_t Vloc, int64_t ld, int64_t v0, const uint32_t *mask,
                        int64_t mask_ld, const int32_t *rows, int64_t F, int64_t B, const uint32_t *records,
                        int32_t nranks, int32_t kmax, const double *temperature, const int32_t *bracket,
                        uint32_t *entries, double *segments, ms_stream_t stream);
int ms_nucleus_cut(const uint32_t *entries, int32_t nranks, const int64_t *bounds, const int32_t *bracket,
                   const int32_t *rows, int64_t F, int64_t B, const uint32_t *records, int32_t kmax,
                   const double *temperature, const double *top_p, const double *uniforms, uint32_t *cut,
                   ms_stream_t stream);
int ms_nucleus_draw(const void *logits, int dtype, int64_t Vloc, int64_t ld, int64_t v0, const uint32_t *mask,
                    int64_t mask_ld, const int32_t *rows, int64_t F, int64_t B, const uint32_t *records,
                    int32_t nranks, int32_t kmax, const double *temperature, const uint32_t *cut,
                    const uint32_t *entries, const double *segments, int32_t rank, int64_t *out,
                    ms_stream_t stream);

/*
 * JSON-grammar allowed-token mask: bit t of a row is
 * JSONLogitsProcessor.is_valid_prefix(prefix + vocab[t])
 * (miniserve/sampler.py:139-148; the allowed_token_ids(partial, vocab) the
 * reference names at sampler.py:120), with is_valid_prefix's answers as
 * CPython 3.12's json decoder gives them.  No counterpart computes this mask
 * in the reference.
 *
 * A row's parse state (ms_json_state_words() 32-bit words) lives in a
 * caller-owned device buffer [B][words]:
 *   ms_json_init     the state after each row's prefix: text r is
 *                    prefix_bytes[prefix_off[r] .. prefix_off[r+1]) (UTF-8)
 *   ms_json_advance  append token tokens[r] (< 0: nothing) of the vocabulary
 *                    to row r, e.g. the token just sampled
 *   ms_build_json_mask
 *                    mask [B, mask_ld] u32, bit (t & 31) of word (t >> 5) set
 *                    when token t may follow (the layout ms_sample's mask
 *                    takes).  row_status bit 1: some token makes the
 *                    reference raise instead (an integer of more than 4300
 *                    digits, or 9997 nested containers), bit 2: some token
 *                    opens or closes more than 64 containers beyond the row's
 *                    own; those tokens' bits are 0.
 * The vocabulary is vocab_bytes[vocab_off[t] .. vocab_off[t+1]) (UTF-8), with
 * vocab_off an int64 array of V + 1 entries.  B <= 65535 for the mask.
 */
int64_t ms_json_state_words(void);
int ms_json_init(const uint8_t *prefix_bytes, const int64_t *prefix_off, int64_t B, uint32_t *states,
                 ms_stream_t stream);
int ms_json_advance(uint32_t *states, int64_t B, const uint8_t *vocab_bytes, const int64_t *vocab_off,
                    int64_t V, const int64_t *tokens, ms_stream_t stream);
int ms_build_json_mask(const uint32_t *states, int64_t B, const uint8_t *vocab_bytes, const int64_t *vocab_off,
                       int64_t V, uint32_t *mask, int64_t mask_ld, int32_t *row_status, ms_stream_t stream);

/* A fixed-width copy of the vocabulary for ms_build_json_mask_packed, made
 * once per vocabulary: packed [V, 4] u32 (16-byte aligned; token t's first 16
 * bytes, zero-padded), lens [V] (its length, 255 for tokens longer than 16
 * bytes, which the mask reads from vocab_bytes).  Same vocabulary layout as
 * ms_build_json_mask.  An addition to the reference interface (no counterpart
 * in miniserve/sampler.py): a faster equivalent of ms_build_json_mask. */
int ms_json_pack_vocab(const uint8_t *vocab_bytes, const int64_t *vocab_off, int64_t V, uint32_t *packed,
                       uint8_t *lens, ms_stream_t stream);
/* ms_build_json_mask with token bytes from ms_json_pack_vocab's tables; the
 * same mask and row_status. */
int ms_build_json_mask_packed(const uint32_t *states, int64_t B, const uint8_t *vocab_bytes,
                              const int64_t *vocab_off, const uint32_t *packed, const uint8_t *lens, int64_t V,
                              uint32_t *mask, int64_t mask_ld, int32_t *row_status, ms_stream_t stream);

/* The fixed-width copy in a caller-chosen token order: position p holds
 * token order[p] (order: int32 [V] on the device, a permutation of 0..V-1;
 * an entry outside it packs an empty token whose bit is never set).  Sorting
 * the vocabulary by (byte length, bytes) puts tokens that take the same
 * automaton steps in the same warp.  An addition to the reference interface
 * (no counterpart in miniserve/sampler.py). */
int ms_json_pack_vocab_ordered(const uint8_t *vocab_bytes, const int64_t *vocab_off, int64_t V,
                               const int32_t *order, uint32_t *packed, uint8_t *lens, ms_stream_t stream);
/* ms_build_json_mask with ms_json_pack_vocab_ordered's tables and the same
 * order: the same mask (in token order) and row_status.  The first
 * ceil(V/32) words of each row are rewritten; the rest of the row is left
 * alone. */
int ms_build_json_mask_ordered(const uint32_t *states, int64_t B, const uint8_t *vocab_bytes,
                               const int64_t *vocab_off, const uint32_t *packed, const uint8_t *lens,
                               const int32_t *order, int64_t V, uint32_t *mask, int64_t mask_ld,
                               int32_t *row_status, ms_stream_t stream);

/*
 * ms_build_json_mask without any device allocation by anyone: the
 * fixed-width vocabulary copy that ms_build_json_mask_packed reads from
 * caller memory lives here in a device array inside the library (4.25 MB,
 * allocated when the library is loaded and held by every GPU that loads it
 * until the process exits), repacked from vocab_bytes / vocab_off on every
 * call.  For callers that cannot allocate device memory themselves: a
 * runtime that owns the whole device through its own memory pool, or a
 * plugin that has no device allocator it may call.  The caller passes the
 * same inputs and outputs as ms_build_json_mask and gets the same mask and
 * row_status.  V <= 262144 (MS_E_TOO_LARGE beyond).  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) with
 * that device current; make that first call before any stream capture.
 * Every call uses the one array: calls that can overlap on the GPU (other
 * streams, other host threads) race and must be serialized by the caller.
 * No counterpart in the reference (miniserve has no device code); an
 * addition to this library's interface.
 */
int ms_build_json_mask_noalloc(const uint32_t *states, int64_t B, const uint8_t *vocab_bytes,
                               const int64_t *vocab_off, int64_t V, uint32_t *mask, int64_t mask_ld,
                               int32_t *row_status, ms_stream_t stream);

/*
 * The allowed-token bitmask from a logits-processor hook's output.
 * Replaces the hook convention of miniserve/model_runner.py:166-168,214-216
 * (fn(logits[V], generated) -> logits[V], a disallowed token set to -inf,
 * then argmax): `logits` [B, ld] (dtype as in ms_sample) holds what the hook
 * returned, and mask[b, t >> 5] bit (t & 31) is set when logits[b, t] is not
 * -inf (a NaN counts as allowed; the sampler then flags the row
 * MS_ROW_NONFINITE).  The mask feeds ms_sample unchanged.  1 <= B <= 65535,
 * mask_ld >= ceil(V/32); words past ceil(V/32) are not written.
 */
int ms_mask_from_logits(const void *logits, int dtype, int64_t B, int64_t V, int64_t ld, uint32_t *mask,
                        int64_t mask_ld, ms_stream_t stream);

/* Human-readable text for an MS_E_* code. */
const char *ms_error_string(int code);

/* cudaError_t of the most recent failed CUDA call in this thread (0 if none). */
int ms_last_cuda_error(void);

/* Library version, e.g. 100 for 0.1.0. */
int ms_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MSSAMPLE_H */
