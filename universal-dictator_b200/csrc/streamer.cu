// Host-side batched streamer: the B200 form of NemotronStreamer (Sources/DictatorCore/Nemotron/
// NemotronStreamer.swift:16-163). The reference drives one encoder per stream, chunk by chunk, from a serial
// queue; here many streams share one engine and every step runs all streams with a ready chunk as one batched
// encoder pass (ud_step_batch) followed by greedy RNN-T decoding with each stream's carried decoder state.
//
// The chunk walk is runBuffered's (NemotronStreamer.swift:70-91): the first chunk is 1 + 8R mel rows with no
// pre-encode cache (and no subsampled frames dropped by the engine), later chunks are 8 + 8R new rows behind a
// 9-row pre-encode cache, the final chunk is whatever remains (at least 8 rows; 1 for a stream's only chunk)
// and keeps all its valid frames (keepAll). For live input (drainChunks, :109-154) a full chunk runs only once
// more rows or the end have arrived, so the final chunk is recognised as such and the outputs of a stream fed
// row by row equal those of the same stream fed at once.
//
// Only the public C ABI of the engine is used.
#include <cstring>
#include <vector>

#include "ud.h"

namespace ud {
ud_status host_fail(ud_status s, const char* msg);
}

namespace {

constexpr int kPreEncodeCache = 9;   // NemotronSchedule.swift:7-16

struct StreamRec {
    bool used = false, finished = false, last = false;
    const float* mel = nullptr;
    int capacity = 0, avail = 0, idx = 0;
    ud_stream_id slot = -1;
    std::vector<int32_t> tokens;
};

}  // namespace

struct ud_streamer {
    ud_engine* e = nullptr;
    ud_config cfg{};
    int lookahead = 0, decode = 0;
    std::vector<StreamRec> recs;
    std::vector<int> free_ids;
    // per-step scratch, sized for max_batch streams
    std::vector<ud_stream_id> ids;
    std::vector<const float*> mels;
    std::vector<int> rows, keep, frames, ntok, who, next;
    std::vector<float> proj;
    std::vector<int32_t> toks;
    std::vector<ud_streamer_id> just_finished;   // ids that finished in the last step
};

extern "C" {

int ud_chunk_next(int lookahead, int idx, int avail, int last, int* start, int* n_rows, int* keep_all,
                  int* next_idx) {
    if (lookahead < 0 || idx < 0 || avail < idx) return -1;
    const bool first = idx == 0;
    const int size = first ? 1 + 8 * lookahead : 8 + 8 * lookahead;
    int chunk_len, keep;
    if (!last) {
        if (avail - idx <= size) return 0;   // not yet known whether this chunk is the final one
        chunk_len = size;
        keep = 0;
    } else {
        if (idx >= avail) return -1;
        chunk_len = (idx + size < avail ? idx + size : avail) - idx;
        if (chunk_len < (first ? 1 : 8)) return -1;
        keep = idx + size >= avail ? 1 : 0;
    }
    const int cache_start = first ? idx : (idx - kPreEncodeCache > 0 ? idx - kPreEncodeCache : 0);
    if (start) *start = cache_start;
    if (n_rows) *n_rows = (idx - cache_start) + chunk_len;
    if (keep_all) *keep_all = keep;
    if (next_idx) *next_idx = idx + size;
    return 1;
}

ud_status ud_streamer_create(ud_engine* e, int lookahead, int decode, ud_streamer** out) {
    if (!e || !out) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (lookahead < 0) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "negative lookahead");
    ud_config cfg;
    ud_status st = ud_get_config(e, &cfg);
    if (st != UD_OK) return st;
    if (cfg.sub_channels <= 0) return ud::host_fail(UD_ERR_UNSUPPORTED, "the streamer needs a subsampling front end");
    if (decode && cfg.joint_dim <= 0) return ud::host_fail(UD_ERR_UNSUPPORTED, "decode needs an RNN-T head");
    if (lookahead + 1 > cfg.max_chunk_frames)   // a chunk yields lookahead + 1 encoder frames
        return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "lookahead too large for max_chunk_frames");
    ud_streamer* s = new ud_streamer;
    s->e = e;
    s->cfg = cfg;
    s->lookahead = lookahead;
    s->decode = decode ? 1 : 0;
    const size_t B = static_cast<size_t>(cfg.max_batch);
    s->ids.resize(B);
    s->mels.resize(B);
    s->rows.resize(B);
    s->keep.resize(B);
    s->frames.resize(B);
    s->ntok.resize(B);
    s->who.resize(B);
    s->next.resize(B);
    if (!s->decode) s->proj.resize(B * cfg.max_chunk_frames * (cfg.joint_dim > 0 ? cfg.joint_dim : cfg.d_model));
    if (s->decode) s->toks.resize(B * cfg.max_chunk_frames * cfg.max_symbols);
    *out = s;
    return UD_OK;
}

ud_status ud_streamer_destroy(ud_streamer* s) {
    if (!s) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL streamer");
    for (StreamRec& r : s->recs)
        if (r.used && !r.finished && r.slot >= 0) ud_stream_close(s->e, r.slot);
    delete s;
    return UD_OK;
}

ud_status ud_streamer_open(ud_streamer* s, const float* mel, int capacity_rows, ud_streamer_id* out) {
    if (!s || !mel || !out) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (capacity_rows < 1) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "empty mel buffer");
    ud_stream_id slot = -1;
    ud_status st = ud_stream_open(s->e, s->lookahead, &slot);
    if (st != UD_OK) return st;
    int id;
    if (!s->free_ids.empty()) {
        id = s->free_ids.back();
        s->free_ids.pop_back();
    } else {
        id = static_cast<int>(s->recs.size());
        s->recs.emplace_back();
    }
    StreamRec& r = s->recs[id];
    r = StreamRec();
    r.used = true;
    r.mel = mel;
    r.capacity = capacity_rows;
    r.slot = slot;
    *out = id;
    return UD_OK;
}

static StreamRec* rec_of(ud_streamer* s, ud_streamer_id id) {
    if (!s || id < 0 || id >= static_cast<int>(s->recs.size()) || !s->recs[id].used) return nullptr;
    return &s->recs[id];
}

ud_status ud_streamer_push(ud_streamer* s, ud_streamer_id id, int n_rows, int last) {
    StreamRec* r = rec_of(s, id);
    if (!r) return ud::host_fail(UD_ERR_NO_STREAM, "unknown streamer id");
    if (r->last) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "rows pushed after the end of the stream");
    if (n_rows < 0 || r->avail + n_rows > r->capacity)
        return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "pushed rows exceed the stream's buffer");
    r->avail += n_rows;
    r->last = last != 0;
    return UD_OK;
}

ud_status ud_streamer_step(ud_streamer* s, int* n_stepped, int* n_finished) {
    if (!s) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL streamer");
    int n = 0, done = 0;
    const int mel_bins = s->cfg.mel_bins;
    s->just_finished.clear();
    for (int id = 0; id < static_cast<int>(s->recs.size()) && n < s->cfg.max_batch; ++id) {
        StreamRec& r = s->recs[id];
        if (!r.used || r.finished) continue;
        int start, rows, keep, nxt;
        const int c = ud_chunk_next(s->lookahead, r.idx, r.avail, r.last ? 1 : 0, &start, &rows, &keep, &nxt);
        if (c == 0) continue;
        if (c < 0) {   // what remains is too short to encode: the stream ends here
            ud_stream_close(s->e, r.slot);
            r.finished = true;
            s->just_finished.push_back(id);
            ++done;
            continue;
        }
        s->ids[n] = r.slot;
        s->mels[n] = r.mel + static_cast<size_t>(start) * mel_bins;
        s->rows[n] = rows;
        s->keep[n] = keep;
        s->who[n] = id;
        s->next[n] = nxt;
        ++n;
    }
    if (n > 0) {
        ud_status st = ud_step_batch(s->e, n, s->ids.data(), s->mels.data(), s->rows.data(), s->rows.data(),
                                     s->keep.data(), s->decode ? nullptr : s->proj.data(), s->frames.data(),
                                     s->decode ? s->toks.data() : nullptr, s->decode ? s->ntok.data() : nullptr);
        if (st != UD_OK) return st;
        const size_t tok_stride = static_cast<size_t>(s->cfg.max_chunk_frames) * s->cfg.max_symbols;
        for (int i = 0; i < n; ++i) {
            StreamRec& r = s->recs[s->who[i]];
            if (s->decode) {
                const int32_t* t = s->toks.data() + i * tok_stride;
                r.tokens.insert(r.tokens.end(), t, t + s->ntok[i]);
            }
            r.idx = s->next[i];
            if (s->keep[i]) {   // the final chunk: free the engine slot
                ud_stream_close(s->e, r.slot);
                r.finished = true;
                s->just_finished.push_back(s->who[i]);
                ++done;
            }
        }
    }
    if (n_stepped) *n_stepped = n;
    if (n_finished) *n_finished = done;
    return UD_OK;
}

ud_status ud_streamer_finished(ud_streamer* s, ud_streamer_id* out, int cap, int* n) {
    if (!s || !n) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    const int k = static_cast<int>(s->just_finished.size());
    if (out && cap > 0) std::memcpy(out, s->just_finished.data(), sizeof(ud_streamer_id) * static_cast<size_t>(k < cap ? k : cap));
    *n = k;
    return UD_OK;
}

ud_status ud_streamer_tokens(ud_streamer* s, ud_streamer_id id, int32_t* out, int cap, int* n_tokens, int* finished) {
    StreamRec* r = rec_of(s, id);
    if (!r) return ud::host_fail(UD_ERR_NO_STREAM, "unknown streamer id");
    const int n = static_cast<int>(r->tokens.size());
    if (out && cap > 0) std::memcpy(out, r->tokens.data(), sizeof(int32_t) * static_cast<size_t>(n < cap ? n : cap));
    if (n_tokens) *n_tokens = n;
    if (finished) *finished = r->finished ? 1 : 0;
    return UD_OK;
}

ud_status ud_streamer_release(ud_streamer* s, ud_streamer_id id) {
    StreamRec* r = rec_of(s, id);
    if (!r) return ud::host_fail(UD_ERR_NO_STREAM, "unknown streamer id");
    if (!r->finished && r->slot >= 0) ud_stream_close(s->e, r->slot);
    *r = StreamRec();
    s->free_ids.push_back(id);
    return UD_OK;
}

}  // extern "C"
