/*
 * gdn_host.h -- host-side runtime around the GDN layer step.  Pure host code: nothing
 * here touches a device or calls CUDA, so it runs (and is tested) without a GPU.
 *
 *   - Token scheduler: continuous batching with the policy of TokenScheduler
 *     (src/scheduler/scheduler.rs:36-174): a FIFO of waiting requests, up to
 *     `prefill_budget` admissions per step, and a round-robin queue of decoding
 *     sequences from which each step takes up to `max_batch` (front first; unfinished
 *     ones go to the back).  Where the reference calls ModelExecutor::prefill and then
 *     ModelExecutor::decode_batch (src/scheduler/executor.rs:21-49) within one step,
 *     a plan here packs the step's prefill chunks and decode tokens into ONE ragged
 *     call (one cu_seqlens table), so a sequence admitted in step k first decodes in
 *     step k+1.  Long prompts may be split into chunks of `prefill_chunk` tokens.
 *   - Slot allocation: the opaque per-sequence state of the reference
 *     (Sequence::state, src/scheduler/sequence.rs:51-66) becomes a slot of a device
 *     pool.  Admission takes a free slot (the caller resets it, gdn_slot_reset, before
 *     the first chunk runs); finishing returns it.
 *   - Slot-range sharding over GPUs: shard s owns global slots
 *     [s * slots_per_shard, (s + 1) * slots_per_shard); a sequence is admitted on the
 *     shard with the most free slots (ties: lowest shard) and stays there.
 *   - Step packing: gdn_pack_step splits a step's entries into per-shard local-slot and
 *     cu_seqlens tables plus a row map, the inputs of gdn_layer_step on each GPU.
 *
 * Conventions: as gdn.h (GDN_OK or a GDN_E_* code; gdn_last_error() has the message).
 * A scheduler is not thread-safe.
 */
#ifndef GDN_B200_HOST_H
#define GDN_B200_HOST_H

#include <stdint.h>

#include "gdn.h"

#ifdef __cplusplus
extern "C" {
#endif

/* What an entry of a step does. */
#define GDN_ENTRY_DECODE 0        /* one token of a decoding sequence */
#define GDN_ENTRY_PREFILL_FIRST 1 /* first prompt chunk: the slot must be reset before the step */
#define GDN_ENTRY_PREFILL_CONT 2  /* a later prompt chunk */

/* Why a sequence finished (FinishReason, src/scheduler/sequence.rs:84-89). */
#define GDN_FINISH_EOS 0
#define GDN_FINISH_MAX_TOKENS 1

/* One sequence's part of a step.  Entry i owns rows [row0_i, row0_i + n_tokens) of the
 * step's packed input, row0_i = sum of n_tokens over entries before i. */
typedef struct gdn_step_entry {
    uint64_t seq_id;  /* id returned by gdn_sched_enqueue */
    int32_t slot;     /* global slot; shard = slot / slots_per_shard */
    int32_t n_tokens; /* rows of this sequence in the step (1 for a decode entry) */
    int32_t kind;     /* GDN_ENTRY_* */
    int32_t pos;      /* tokens of this sequence processed before this step */
} gdn_step_entry;

/* Packs one step into per-shard ragged tables, shard-major (entries keep their order
 * inside a shard).  Caller-allocated outputs:
 *   shard_n_seq[n_shards], shard_n_tokens[n_shards]
 *   slot_ids[n_entries]                local slot ids; shard s's block starts at
 *                                      sum_{r<s} shard_n_seq[r]
 *   cu_seqlens[n_entries + n_shards]   shard s's table (shard_n_seq[s] + 1 entries,
 *                                      starting at 0) starts at sum_{r<s} (shard_n_seq[r] + 1)
 *   row_src[sum of n_tokens]           shard-major packed row -> row of the step's input
 * Errors: GDN_E_INVALID (NULL, n_tokens < 1, bad shard geometry), GDN_E_BAD_SLOT (a slot
 * outside [0, n_shards * slots_per_shard) or used by two entries). */
GDN_API int gdn_pack_step(const gdn_step_entry* entries, int32_t n_entries, int32_t n_shards,
                          int32_t slots_per_shard, int32_t* shard_n_seq, int32_t* shard_n_tokens,
                          int32_t* slot_ids, int32_t* cu_seqlens, int32_t* row_src);

typedef struct gdn_sched gdn_sched;

typedef struct gdn_sched_config {
    int32_t n_shards;        /* GPUs (>= 1) */
    int32_t slots_per_shard; /* pool slots per GPU (>= 1) */
    int32_t max_batch;       /* decoding sequences per step (max_batch_size, >= 1) */
    int32_t prefill_budget;  /* new sequences admitted per step (>= 0; the reference's default is 1) */
    int32_t prefill_chunk;   /* prompt tokens per sequence per step; 0 = the whole prompt */
} gdn_sched_config;

/* SchedulerStats (src/scheduler/scheduler.rs:16-23), plus the pool view. */
typedef struct gdn_sched_stats {
    uint64_t total_requests;   /* enqueued so far */
    uint64_t tokens_generated; /* decode tokens (the first token of a prefill is not counted) */
    uint64_t iterations;       /* steps that ran a decode batch */
    int32_t active;            /* decoding sequences */
    int32_t waiting;           /* not yet admitted */
    int32_t prefilling;        /* admitted, prompt not finished */
    int32_t free_slots;        /* over all shards */
} gdn_sched_stats;

GDN_API int gdn_sched_create(const gdn_sched_config* cfg, gdn_sched** out);
GDN_API int gdn_sched_destroy(gdn_sched* s);

/* Enqueue a request (TokenScheduler::enqueue).  prompt_len >= 1, max_tokens >= 1. */
GDN_API int gdn_sched_enqueue(gdn_sched* s, int32_t prompt_len, int32_t max_tokens, uint64_t* id);

/* Plan the next step into entries[0..cap): first the next chunk of every prompt in progress,
 * then up to prefill_budget admissions (stopping early when no slot is free), then up to
 * max_batch decode entries from the front of the round-robin queue.  *n_entries may be 0.
 * GDN_E_INVALID if the previous plan has not been completed or cap is too small. */
GDN_API int gdn_sched_plan(gdn_sched* s, gdn_step_entry* entries, int32_t cap, int32_t* n_entries);

/* Complete the planned step.  stop[i] != 0: the token entry i produced is an end token
 * (Sequence::should_stop's eos test); ignored for chunks that do not end a prompt.  A prompt's
 * last chunk yields the first token (tokens_generated = 1); each decode entry one more.
 * Finished sequences release their slot and are queued for gdn_sched_drain_finished. */
GDN_API int gdn_sched_complete(gdn_sched* s, const uint8_t* stop);

/* Up to cap finished (id, GDN_FINISH_*) pairs, oldest first; *n receives the count. */
GDN_API int gdn_sched_drain_finished(gdn_sched* s, uint64_t* ids, int32_t* reasons, int32_t cap, int32_t* n);

GDN_API int gdn_sched_stats_get(const gdn_sched* s, gdn_sched_stats* out);

/* The decoding queue front to back (up to cap ids). */
GDN_API int gdn_sched_active_ids(const gdn_sched* s, uint64_t* ids, int32_t cap, int32_t* n);

/* Free slots of one shard. */
GDN_API int gdn_sched_free_slots(const gdn_sched* s, int32_t shard, int32_t* n);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_HOST_H */
