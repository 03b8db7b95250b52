// gdn_host.cpp -- host runtime around the GDN step: token scheduler, slot allocation,
// slot-range sharding and step packing (the C ABI of include/gdn_host.h).  No device code.
//
// Scheduling policy follows TokenScheduler::step (src/scheduler/scheduler.rs:96-174):
// waiting requests are admitted FIFO, at most prefill_budget per step; the decode batch is
// the front max_batch of the active queue; after the step, sequences whose prompt finished
// join the back of the active queue first, then unfinished decoders are requeued at the
// back (round-robin fairness); a prompt's last chunk yields the first token
// (tokens_generated = 1, not counted in the decode-token statistic); a sequence stops on an
// end token or when tokens_generated reaches max_tokens (Sequence::should_stop,
// src/scheduler/sequence.rs:127-131).  A stop at the end of a prompt is reported as
// GDN_FINISH_EOS whatever its cause, as the reference's prefill path does (scheduler.rs:110-113).
#include <algorithm>
#include <deque>
#include <new>
#include <vector>

#include "gdn_host.h"
#include "gdn_internal.h"

namespace {

struct Seq {
    uint64_t id;
    int32_t prompt_len;
    int32_t max_tokens;
    int32_t slot = -1;
    int32_t pos = 0;               // prompt tokens processed
    int32_t tokens_generated = 0;  // first token counts 1
};

struct Planned {
    Seq* seq;
    int32_t kind;
    int32_t n_tokens;
};

}  // namespace

struct gdn_sched {
    gdn_sched_config cfg;
    uint64_t next_id = 1;
    std::deque<Seq*> waiting;     // FIFO
    std::deque<Seq*> prefilling;  // admitted, prompt in progress (FIFO)
    std::deque<Seq*> active;      // round-robin decode queue
    std::vector<std::vector<int32_t>> free_slots;  // per shard, a stack (lowest slot on top)
    std::vector<Planned> plan;
    bool planned = false;
    std::deque<std::pair<uint64_t, int32_t>> finished;
    gdn_sched_stats stats{};
};

namespace {

void release(gdn_sched* s, Seq* q, int32_t reason) {
    const int32_t shard = q->slot / s->cfg.slots_per_shard;
    s->free_slots[shard].push_back(q->slot - shard * s->cfg.slots_per_shard);
    s->finished.emplace_back(q->id, reason);
    delete q;
}

void refresh(gdn_sched* s) {
    s->stats.active = (int32_t)s->active.size();
    s->stats.waiting = (int32_t)s->waiting.size();
    s->stats.prefilling = (int32_t)s->prefilling.size();
    int32_t f = 0;
    for (const auto& v : s->free_slots) f += (int32_t)v.size();
    s->stats.free_slots = f;
}

// Shard with the most free slots (ties: lowest index); -1 when every shard is full.
int32_t pick_shard(const gdn_sched* s) {
    int32_t best = -1;
    size_t most = 0;
    for (int32_t i = 0; i < (int32_t)s->free_slots.size(); ++i)
        if (s->free_slots[i].size() > most) {
            most = s->free_slots[i].size();
            best = i;
        }
    return best;
}

}  // namespace

extern "C" {

int gdn_pack_step(const gdn_step_entry* e, int32_t n, int32_t n_shards, int32_t per, int32_t* shard_n_seq,
                  int32_t* shard_n_tokens, int32_t* slot_ids, int32_t* cu, int32_t* row_src) {
    using gdn::record_error;
    if (n < 0 || n_shards < 1 || per < 1) return record_error(GDN_E_INVALID, "bad step size or shard geometry");
    if (!shard_n_seq || !shard_n_tokens || !cu || (n > 0 && (!e || !slot_ids || !row_src)))
        return record_error(GDN_E_INVALID, "NULL argument");
    const long long total_slots = (long long)n_shards * per;
    std::vector<int32_t> seen;
    seen.reserve(n);
    for (int32_t i = 0; i < n; ++i) {
        if (e[i].n_tokens < 1) return record_error(GDN_E_INVALID, "an entry has n_tokens < 1");
        if (e[i].slot < 0 || e[i].slot >= total_slots) return record_error(GDN_E_BAD_SLOT, "slot outside the shards");
        seen.push_back(e[i].slot);
    }
    std::sort(seen.begin(), seen.end());
    if (std::adjacent_find(seen.begin(), seen.end()) != seen.end())
        return record_error(GDN_E_BAD_SLOT, "a slot is used by two entries of one step");
    // global row offset of every entry
    std::vector<long long> row0(n);
    long long r = 0;
    for (int32_t i = 0; i < n; ++i) {
        row0[i] = r;
        r += e[i].n_tokens;
    }
    if (r > INT32_MAX) return record_error(GDN_E_INVALID, "step has more than 2^31 rows");
    int32_t seq_base = 0, cu_base = 0, row_base = 0;
    for (int32_t s = 0; s < n_shards; ++s) {
        int32_t ns = 0, nt = 0;
        cu[cu_base] = 0;
        for (int32_t i = 0; i < n; ++i) {
            if (e[i].slot / per != s) continue;
            slot_ids[seq_base + ns] = e[i].slot - s * per;
            for (int32_t t = 0; t < e[i].n_tokens; ++t) row_src[row_base + nt + t] = (int32_t)(row0[i] + t);
            nt += e[i].n_tokens;
            ++ns;
            cu[cu_base + ns] = nt;
        }
        shard_n_seq[s] = ns;
        shard_n_tokens[s] = nt;
        seq_base += ns;
        cu_base += ns + 1;
        row_base += nt;
    }
    return gdn::record_ok();
}

int gdn_sched_create(const gdn_sched_config* cfg, gdn_sched** out) {
    using gdn::record_error;
    if (!cfg || !out) return record_error(GDN_E_INVALID, "NULL argument");
    *out = nullptr;
    if (cfg->n_shards < 1 || cfg->slots_per_shard < 1 || cfg->max_batch < 1 || cfg->prefill_budget < 0 ||
        cfg->prefill_chunk < 0)
        return record_error(GDN_E_INVALID, "scheduler config out of range");
    gdn_sched* s = new (std::nothrow) gdn_sched();
    if (!s) return record_error(GDN_E_NOMEM, "host allocation failed");
    s->cfg = *cfg;
    s->free_slots.resize(cfg->n_shards);
    for (auto& v : s->free_slots) {
        v.reserve(cfg->slots_per_shard);
        for (int32_t i = cfg->slots_per_shard - 1; i >= 0; --i) v.push_back(i);
    }
    refresh(s);
    *out = s;
    return gdn::record_ok();
}

int gdn_sched_destroy(gdn_sched* s) {
    if (!s) return gdn::record_ok();
    for (auto* q : s->waiting) delete q;
    for (auto* q : s->prefilling) delete q;
    for (auto* q : s->active) delete q;
    delete s;
    return gdn::record_ok();
}

int gdn_sched_enqueue(gdn_sched* s, int32_t prompt_len, int32_t max_tokens, uint64_t* id) {
    using gdn::record_error;
    if (!s || !id) return record_error(GDN_E_INVALID, "NULL argument");
    if (prompt_len < 1 || max_tokens < 1) return record_error(GDN_E_INVALID, "prompt_len and max_tokens must be >= 1");
    Seq* q = new (std::nothrow) Seq();
    if (!q) return record_error(GDN_E_NOMEM, "host allocation failed");
    q->id = s->next_id++;
    q->prompt_len = prompt_len;
    q->max_tokens = max_tokens;
    s->waiting.push_back(q);
    s->stats.total_requests += 1;
    refresh(s);
    *id = q->id;
    return gdn::record_ok();
}

int gdn_sched_plan(gdn_sched* s, gdn_step_entry* entries, int32_t cap, int32_t* n_entries) {
    using gdn::record_error;
    if (!s || !n_entries || cap < 0 || (cap > 0 && !entries)) return record_error(GDN_E_INVALID, "NULL argument");
    if (s->planned) return record_error(GDN_E_INVALID, "the previous plan has not been completed");
    const int32_t chunk = s->cfg.prefill_chunk;
    auto take = [&](Seq* q) {
        const int32_t left = q->prompt_len - q->pos;
        return chunk > 0 && chunk < left ? chunk : left;
    };
    std::vector<Planned> plan;
    for (Seq* q : s->prefilling) plan.push_back({q, GDN_ENTRY_PREFILL_CONT, take(q)});
    // admissions: a slot each, FIFO, stop at the budget or when the pool is full
    std::vector<Seq*> admitted;
    for (int32_t k = 0; k < s->cfg.prefill_budget && k < (int32_t)s->waiting.size(); ++k) {
        const int32_t shard = pick_shard(s);
        if (shard < 0) break;
        Seq* q = s->waiting[k];
        q->slot = shard * s->cfg.slots_per_shard + s->free_slots[shard].back();
        s->free_slots[shard].pop_back();
        admitted.push_back(q);
        plan.push_back({q, GDN_ENTRY_PREFILL_FIRST, take(q)});
    }
    const int32_t batch = std::min<int32_t>(s->cfg.max_batch, (int32_t)s->active.size());
    for (int32_t k = 0; k < batch; ++k) plan.push_back({s->active[k], GDN_ENTRY_DECODE, 1});
    if ((int32_t)plan.size() > cap) {
        // undo the admissions' slot grabs
        for (Seq* q : admitted) {
            const int32_t shard = q->slot / s->cfg.slots_per_shard;
            s->free_slots[shard].push_back(q->slot - shard * s->cfg.slots_per_shard);
            q->slot = -1;
        }
        return record_error(GDN_E_INVALID, "entries buffer too small for the step");
    }
    for (size_t k = 0; k < admitted.size(); ++k) s->waiting.pop_front();
    for (Seq* q : admitted) s->prefilling.push_back(q);
    for (size_t i = 0; i < plan.size(); ++i) {
        const Planned& p = plan[i];
        const int32_t pos = p.kind == GDN_ENTRY_DECODE ? p.seq->prompt_len + p.seq->tokens_generated - 1 : p.seq->pos;
        entries[i] = gdn_step_entry{p.seq->id, p.seq->slot, p.n_tokens, p.kind, pos};
    }
    s->plan = std::move(plan);
    s->planned = true;
    *n_entries = (int32_t)s->plan.size();
    refresh(s);
    return gdn::record_ok();
}

int gdn_sched_complete(gdn_sched* s, const uint8_t* stop) {
    using gdn::record_error;
    if (!s) return record_error(GDN_E_INVALID, "NULL argument");
    if (!s->planned) return record_error(GDN_E_INVALID, "no planned step to complete");
    if (!s->plan.empty() && !stop) return record_error(GDN_E_INVALID, "stop flags are NULL");
    // the prefill entries lead the plan and the decode batch is the active front, in order
    std::deque<Seq*> still_prefilling;
    int32_t n_decode = 0;
    for (size_t i = 0; i < s->plan.size(); ++i) {
        const Planned& p = s->plan[i];
        Seq* q = p.seq;
        if (p.kind == GDN_ENTRY_DECODE) {
            ++n_decode;
            continue;
        }
        q->pos += p.n_tokens;
        if (q->pos < q->prompt_len) {
            still_prefilling.push_back(q);
            continue;
        }
        q->tokens_generated = 1;
        if (stop[i] || q->tokens_generated >= q->max_tokens)
            release(s, q, GDN_FINISH_EOS);
        else
            s->active.push_back(q);
    }
    s->prefilling.swap(still_prefilling);
    // the decode batch is the first n_decode of the active queue (prefills completed above were
    // appended behind it); take it off the front, then requeue its unfinished members
    s->active.erase(s->active.begin(), s->active.begin() + n_decode);
    for (size_t i = 0; i < s->plan.size(); ++i) {
        if (s->plan[i].kind != GDN_ENTRY_DECODE) continue;
        Seq* q = s->plan[i].seq;
        q->tokens_generated += 1;
        s->stats.tokens_generated += 1;
        if (stop[i])
            release(s, q, GDN_FINISH_EOS);
        else if (q->tokens_generated >= q->max_tokens)
            release(s, q, GDN_FINISH_MAX_TOKENS);
        else
            s->active.push_back(q);
    }
    if (n_decode > 0) s->stats.iterations += 1;
    s->plan.clear();
    s->planned = false;
    refresh(s);
    return gdn::record_ok();
}

int gdn_sched_drain_finished(gdn_sched* s, uint64_t* ids, int32_t* reasons, int32_t cap, int32_t* n) {
    using gdn::record_error;
    if (!s || !n || cap < 0 || (cap > 0 && (!ids || !reasons))) return record_error(GDN_E_INVALID, "NULL argument");
    int32_t k = 0;
    while (k < cap && !s->finished.empty()) {
        ids[k] = s->finished.front().first;
        reasons[k] = s->finished.front().second;
        s->finished.pop_front();
        ++k;
    }
    *n = k;
    return gdn::record_ok();
}

int gdn_sched_stats_get(const gdn_sched* s, gdn_sched_stats* out) {
    if (!s || !out) return gdn::record_error(GDN_E_INVALID, "NULL argument");
    *out = s->stats;
    return gdn::record_ok();
}

int gdn_sched_active_ids(const gdn_sched* s, uint64_t* ids, int32_t cap, int32_t* n) {
    if (!s || !n || cap < 0 || (cap > 0 && !ids)) return gdn::record_error(GDN_E_INVALID, "NULL argument");
    int32_t k = 0;
    for (const Seq* q : s->active) {
        if (k >= cap) break;
        ids[k++] = q->id;
    }
    *n = k;
    return gdn::record_ok();
}

int gdn_sched_free_slots(const gdn_sched* s, int32_t shard, int32_t* n) {
    if (!s || !n) return gdn::record_error(GDN_E_INVALID, "NULL argument");
    if (shard < 0 || shard >= s->cfg.n_shards) return gdn::record_error(GDN_E_INVALID, "shard out of range");
    *n = (int32_t)s->free_slots[shard].size();
    return gdn::record_ok();
}

}  // extern "C"
