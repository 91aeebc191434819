// Host-side batched streamer: the B200 form of NemotronStreamer (Sources/DictatorCore/Nemotron/
// NemotronStreamer.swift:16-163). The reference drives one encoder per stream, chunk by chunk, from a serial
// queue; here many streams share one engine and every step runs all streams with a ready chunk as one batched
// encoder pass (ud_step_batch) followed by greedy RNN-T decoding with each stream's carried decoder state.
//
// The chunk walk is the live one, drainChunks (NemotronStreamer.swift:109-154): the first chunk is 1 + 8R mel
// rows with no pre-encode cache (and no subsampled frames dropped by the engine), later chunks are 8 + 8R new
// rows behind a 9-row pre-encode cache, each run as soon as its rows exist; at the end the rest runs as the final
// chunk (keepAll), a tail shorter than the minimum chunk (8 rows; 1 for a stream's only chunk) zero-extended to
// it and masked when end padding is on (the reference's default, endPadding :29-31) or dropped when it is off
// (NeMo's batch-1 schedule and runBuffered, :70-91). Over a complete buffer without end padding the walk is
// runBuffered's, and a stream fed row by row gives the chunks of the same stream fed at once.
//
// Streams take mel rows from a caller-owned buffer (ud_streamer_open / ud_streamer_push), or audio through the
// GPU mel frontend (ud_streamer_open_audio / ud_streamer_push_audio: NemotronStreamer.push(samples:) and
// flush(), :95-107), whose rows the streamer keeps only as far back as the pre-encode cache needs.
//
// Only the public C ABI of the engine and the mel frontend is used.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstddef>
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
    bool final_issued = false;      // pipelined: the final chunk is in flight
    const float* mel = nullptr;     // caller-owned rows [capacity, mel_bins] (mel streams)
    int capacity = 0, avail = 0, idx = 0;
    ud_stream_id slot = -1;
    std::vector<int32_t> tokens;
    // per token: the input received when its step ran and that step's wall seconds (Emission); per step the
    // stream took part in: the step's wall seconds (wallTimes)
    int64_t samples = 0;            // audio samples pushed (audio streams)
    std::vector<int64_t> emit_samples;
    std::vector<double> emit_secs, step_secs;
    // audio streams: the frontend's stream and the rows kept from row `own_start` on
    int mel_id = -1;
    std::vector<float> own;
    int own_start = 0;
};

}  // namespace

struct ud_streamer {
    ud_engine* e = nullptr;
    ud_config cfg{};
    int lookahead = 0, decode = 0;
    std::vector<StreamRec> recs;
    std::vector<int> free_ids;
    // per-step scratch, sized for max_batch streams
    int end_padding = 1;
    ud_mel* mel = nullptr;          // the frontend of the audio streams (all of them use one)
    std::vector<ud_stream_id> ids;
    std::vector<const float*> mels;
    std::vector<int> rows, valid, keep, frames, ntok, who, next;
    std::vector<float> pad;         // padded final tails, max_batch x (9 + 8) rows
    std::vector<float> proj;
    std::vector<int32_t> toks;
    std::vector<ud_streamer_id> just_finished;   // ids that finished in the last step
    std::vector<ud_streamer_id> carry;           // finished by a release between steps: reported by the next step
    // Pipelined mode (ud_streamer_set_pipelined): chunk rows staged in pinned buffers at a fixed stride, tokens
    // copied back into pinned buffers, both double-buffered; a step's results are taken in by the next call.
    int pipelined = 0;
    int buf = 0;
    size_t stage_rows = 0;
    float* stage[2] = {};
    int32_t* ptoks[2] = {};
    int* pntok[2] = {};
    struct Pending {
        bool active = false;
        int b = 0;
        std::vector<int> who, keep;
        std::vector<int64_t> seen;
        std::chrono::steady_clock::time_point t0;
    } pend;
};

extern "C" {

int ud_chunk_next(int lookahead, int idx, int avail, int last, int end_padding, int* start, int* n_rows,
                  int* valid_rows, int* keep_all, int* next_idx) {
    if (lookahead < 0 || idx < 0 || avail < idx) return -1;
    const bool first = idx == 0;
    const int size = first ? 1 + 8 * lookahead : 8 + 8 * lookahead;
    const int end = idx + size;
    if (end > avail && !last) return 0;   // the chunk's rows are not all here yet
    const int chunk_end = end < avail ? end : avail;
    const int chunk_len = chunk_end - idx;
    const int min_len = first ? 1 : 8;
    if (chunk_len <= 0 || (chunk_len < min_len && !end_padding)) return -1;   // the stream has ended
    const int cache_start = first ? idx : (idx - kPreEncodeCache > 0 ? idx - kPreEncodeCache : 0);
    const int rows = chunk_end - cache_start;
    const int pad = chunk_len < min_len ? min_len - chunk_len : 0;   // zero rows of a short final tail
    if (start) *start = cache_start;
    if (n_rows) *n_rows = rows + pad;
    if (valid_rows) *valid_rows = rows;
    if (keep_all) *keep_all = (pad > 0 || (last && end >= avail)) ? 1 : 0;
    if (next_idx) *next_idx = end;
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
    s->valid.resize(B);
    s->keep.resize(B);
    s->pad.resize(B * (kPreEncodeCache + 8) * static_cast<size_t>(cfg.mel_bins));
    s->frames.resize(B);
    s->ntok.resize(B);
    s->who.resize(B);
    s->next.resize(B);
    if (!s->decode) s->proj.resize(B * cfg.max_chunk_frames * (cfg.joint_dim > 0 ? cfg.joint_dim : cfg.d_model));
    if (s->decode) s->toks.resize(B * cfg.max_chunk_frames * cfg.max_symbols);
    *out = s;
    return UD_OK;
}

ud_status ud_streamer_set_end_padding(ud_streamer* s, int on) {
    if (!s) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL streamer");
    s->end_padding = on ? 1 : 0;
    return UD_OK;
}

ud_status ud_streamer_destroy(ud_streamer* s) {
    if (!s) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL streamer");
    if (s->pend.active) ud_step_sync(s->e);   // the step in flight reads the pinned stage
    for (StreamRec& r : s->recs) {
        if (r.used && !r.finished && r.slot >= 0) ud_stream_close(s->e, r.slot);
        if (r.used && r.mel_id >= 0 && s->mel) ud_mel_stream_close(s->mel, r.mel_id);
    }
    for (int b = 0; b < 2; ++b) {
        if (s->stage[b]) cudaFreeHost(s->stage[b]);
        if (s->ptoks[b]) cudaFreeHost(s->ptoks[b]);
        if (s->pntok[b]) cudaFreeHost(s->pntok[b]);
    }
    delete s;
    return UD_OK;
}

static ud_status open_rec(ud_streamer* s, ud_streamer_id* out) {
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
    r.slot = slot;
    *out = id;
    return UD_OK;
}

ud_status ud_streamer_open(ud_streamer* s, const float* mel, int capacity_rows, ud_streamer_id* out) {
    if (!s || !mel || !out) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (capacity_rows < 1) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "empty mel buffer");
    ud_status st = open_rec(s, out);
    if (st != UD_OK) return st;
    StreamRec& r = s->recs[*out];
    r.mel = mel;
    r.capacity = capacity_rows;
    return UD_OK;
}

ud_status ud_streamer_open_audio(ud_streamer* s, ud_mel* mel, ud_streamer_id* out) {
    if (!s || !mel || !out) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (s->mel && s->mel != mel) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "a streamer's audio streams share one frontend");
    int mid = -1;
    ud_status st = ud_mel_stream_open(mel, &mid);
    if (st != UD_OK) return st;
    st = open_rec(s, out);
    if (st != UD_OK) {
        ud_mel_stream_close(mel, mid);
        return st;
    }
    s->mel = mel;
    s->recs[*out].mel_id = mid;
    return UD_OK;
}

static StreamRec* rec_of(ud_streamer* s, ud_streamer_id id) {
    if (!s || id < 0 || id >= static_cast<int>(s->recs.size()) || !s->recs[id].used) return nullptr;
    return &s->recs[id];
}

ud_status ud_streamer_push_audio(ud_streamer* s, int n, const ud_streamer_id* ids, const float* const* samples,
                                 const int* n_samples, const int* last) {
    if (!s || n < 0 || (n > 0 && (!ids || !samples || !n_samples))) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (n == 0) return UD_OK;
    std::vector<int> mids(static_cast<size_t>(n)), fin(static_cast<size_t>(n)), frames(static_cast<size_t>(n));
    int cap = 1;
    for (int i = 0; i < n; ++i) {
        StreamRec* r = rec_of(s, ids[i]);
        if (!r) return ud::host_fail(UD_ERR_NO_STREAM, "unknown streamer id");
        if (r->last) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "audio pushed after the end of the stream");
        if (r->mel_id < 0) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "not an audio stream");
        for (int j = 0; j < i; ++j)
            if (ids[j] == ids[i]) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "a stream appears twice in one push");
        if (n_samples[i] < 0) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "negative sample count");
        mids[i] = r->mel_id;
        fin[i] = last && last[i] ? 1 : 0;
        cap = std::max(cap, n_samples[i] / 160 + 4);   // frames one push can complete (hop 160)
    }
    const size_t bins = static_cast<size_t>(s->cfg.mel_bins);
    std::vector<float> out(static_cast<size_t>(n) * cap * bins);
    ud_status st = ud_mel_push_batch(s->mel, n, mids.data(), samples, n_samples, fin.data(), out.data(), cap,
                                     frames.data());
    if (st != UD_OK) return st;
    for (int i = 0; i < n; ++i) {
        StreamRec& r = s->recs[ids[i]];
        const float* f = out.data() + static_cast<size_t>(i) * cap * bins;
        r.own.insert(r.own.end(), f, f + static_cast<size_t>(frames[i]) * bins);
        r.avail += frames[i];
        r.samples += n_samples[i];
        if (fin[i]) r.last = true;
    }
    return UD_OK;
}

ud_status ud_streamer_push(ud_streamer* s, ud_streamer_id id, int n_rows, int last) {
    StreamRec* r = rec_of(s, id);
    if (!r) return ud::host_fail(UD_ERR_NO_STREAM, "unknown streamer id");
    if (r->mel_id >= 0) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "an audio stream takes ud_streamer_push_audio");
    if (r->last) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "rows pushed after the end of the stream");
    if (n_rows < 0 || r->avail + n_rows > r->capacity)
        return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "pushed rows exceed the stream's buffer");
    r->avail += n_rows;
    r->last = last != 0;
    return UD_OK;
}

// Frees a finished stream's engine slot and frontend stream.
static void finish_rec(ud_streamer* s, StreamRec& r, int id, int* done) {
    ud_stream_close(s->e, r.slot);
    if (r.mel_id >= 0) {
        ud_mel_stream_close(s->mel, r.mel_id);
        r.mel_id = -2;   // an audio stream whose frontend stream is closed
        std::vector<float>().swap(r.own);
    }
    r.finished = true;
    s->just_finished.push_back(id);
    ++*done;
}

// Keeps only the pre-encode cache window of an audio stream's rows.
static void trim_audio(ud_streamer* s, StreamRec& r) {
    const size_t bins = static_cast<size_t>(s->cfg.mel_bins);
    const int keep_from = r.idx - kPreEncodeCache;
    if (r.mel_id >= 0 && keep_from > r.own_start) {
        const size_t drop = std::min(r.own.size(), static_cast<size_t>(keep_from - r.own_start) * bins);
        r.own.erase(r.own.begin(), r.own.begin() + static_cast<std::ptrdiff_t>(drop));
        r.own_start = keep_from;
    }
}

// Appends one completed step's tokens and records to its streams; finishes those whose final chunk it was.
static void take_results(ud_streamer* s, int n, const int* who, const int* keep, const int64_t* seen,
                         const int32_t* toks, const int* ntok, double dt, int* done) {
    const size_t tok_stride = static_cast<size_t>(s->cfg.max_chunk_frames) * s->cfg.max_symbols;
    for (int i = 0; i < n; ++i) {
        StreamRec& r = s->recs[who[i]];
        if (s->decode) {
            const int32_t* t = toks + i * tok_stride;
            r.tokens.insert(r.tokens.end(), t, t + ntok[i]);
            r.emit_samples.insert(r.emit_samples.end(), static_cast<size_t>(ntok[i]), seen[i]);
            r.emit_secs.insert(r.emit_secs.end(), static_cast<size_t>(ntok[i]), dt);
        }
        r.step_secs.push_back(dt);
        if (keep[i]) finish_rec(s, r, who[i], done);
    }
}

// Pipelined mode: takes in the results of the step in flight (its device work is complete).
static void take_pending(ud_streamer* s, int* done) {
    ud_streamer::Pending& p = s->pend;
    if (!p.active) return;
    const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - p.t0).count();
    take_results(s, static_cast<int>(p.who.size()), p.who.data(), p.keep.data(), p.seen.data(), s->ptoks[p.b],
                 s->pntok[p.b], dt, done);
    p.active = false;
}

static ud_status pipeline_setup(ud_streamer* s) {
    if (s->stage[0]) return UD_OK;
    const size_t B = static_cast<size_t>(s->cfg.max_batch);
    s->stage_rows = static_cast<size_t>(kPreEncodeCache + 8 + 8 * s->lookahead);   // the longest chunk
    const size_t tok_n = B * s->cfg.max_chunk_frames * s->cfg.max_symbols;
    for (int b = 0; b < 2; ++b) {
        if (cudaMallocHost(&s->stage[b], sizeof(float) * B * s->stage_rows * s->cfg.mel_bins) != cudaSuccess ||
            cudaMallocHost(&s->ptoks[b], sizeof(int32_t) * (tok_n > 0 ? tok_n : 1)) != cudaSuccess ||
            cudaMallocHost(&s->pntok[b], sizeof(int) * B) != cudaSuccess) {
            cudaGetLastError();
            return ud::host_fail(UD_ERR_OUT_OF_MEMORY, "pinned streamer staging");
        }
    }
    return UD_OK;
}

ud_status ud_streamer_set_pipelined(ud_streamer* s, int on) {
    if (!s) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL streamer");
    if (!on && s->pipelined) {   // complete the step in flight before leaving the mode
        ud_status st = ud_step_sync(s->e);
        if (st != UD_OK) return st;
        int done = 0;
        take_pending(s, &done);
    }
    if (on) {
        if (!s->decode) return ud::host_fail(UD_ERR_UNSUPPORTED, "the pipelined streamer decodes");
        ud_status st = pipeline_setup(s);
        if (st != UD_OK) return st;
    }
    s->pipelined = on ? 1 : 0;
    return UD_OK;
}

ud_status ud_streamer_step(ud_streamer* s, int* n_stepped, int* n_finished) {
    if (!s) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL streamer");
    int n = 0, done = 0;
    const size_t bins = static_cast<size_t>(s->cfg.mel_bins);
    const size_t pad_rows = kPreEncodeCache + 8;
    const bool pipe = s->pipelined != 0;
    const int sb = s->buf;
    std::vector<int64_t> seen;
    s->just_finished.swap(s->carry);
    s->carry.clear();
    for (int id = 0; id < static_cast<int>(s->recs.size()) && n < s->cfg.max_batch; ++id) {
        StreamRec& r = s->recs[id];
        if (!r.used || r.finished || r.final_issued) continue;
        int start, rows, valid, keep, nxt;
        const int c = ud_chunk_next(s->lookahead, r.idx, r.avail, r.last ? 1 : 0, s->end_padding, &start, &rows,
                                    &valid, &keep, &nxt);
        if (c == 0) continue;
        if (c < 0) {   // nothing left, or a tail too short to encode without end padding: the stream ends here
            finish_rec(s, r, id, &done);
            continue;
        }
        const float* src = r.mel_id != -1 ? r.own.data() + static_cast<size_t>(start - r.own_start) * bins
                                          : r.mel + static_cast<size_t>(start) * bins;
        if (pipe) {   // the rows into the pinned stage at a fixed stride, a padded tail's zero rows included
            float* dst = s->stage[sb] + static_cast<size_t>(n) * s->stage_rows * bins;
            std::memcpy(dst, src, sizeof(float) * valid * bins);
            if (rows > valid) std::memset(dst + static_cast<size_t>(valid) * bins, 0, sizeof(float) * (rows - valid) * bins);
            src = dst;
        } else if (rows > valid) {   // a padded final tail: the valid rows, then zero rows
            float* dst = s->pad.data() + static_cast<size_t>(n) * pad_rows * bins;
            std::memcpy(dst, src, sizeof(float) * valid * bins);
            std::memset(dst + static_cast<size_t>(valid) * bins, 0, sizeof(float) * (rows - valid) * bins);
            src = dst;
        }
        s->ids[n] = r.slot;
        s->mels[n] = src;
        s->rows[n] = rows;
        s->valid[n] = valid;
        s->keep[n] = keep;
        s->who[n] = id;
        s->next[n] = nxt;
        seen.push_back(r.mel_id != -1 ? r.samples : static_cast<int64_t>(r.avail) * 160);
        ++n;
    }
    if (pipe) {
        // Issue this step; the call returns once the step before it is complete, whose results are taken in.
        if (n > 0) {
            const auto t0 = std::chrono::steady_clock::now();
            ud_status st = ud_step_batch_async(s->e, n, s->ids.data(), s->mels.data(), s->rows.data(),
                                               s->valid.data(), s->keep.data(), nullptr, s->frames.data(),
                                               s->ptoks[sb], s->pntok[sb]);
            if (st != UD_OK) return st;
            take_pending(s, &done);
            ud_streamer::Pending& p = s->pend;
            p.active = true;
            p.b = sb;
            p.who.assign(s->who.begin(), s->who.begin() + n);
            p.keep.assign(s->keep.begin(), s->keep.begin() + n);
            p.seen = seen;
            p.t0 = t0;
            s->buf ^= 1;
            for (int i = 0; i < n; ++i) {
                StreamRec& r = s->recs[s->who[i]];
                r.idx = s->next[i];
                if (s->keep[i]) r.final_issued = true;
                else trim_audio(s, r);   // the chunk's rows are in the stage already
            }
        } else if (s->pend.active) {
            ud_status st = ud_step_sync(s->e);
            if (st != UD_OK) return st;
            take_pending(s, &done);
        }
    } else if (n > 0) {
        const auto t0 = std::chrono::steady_clock::now();
        ud_status st = ud_step_batch(s->e, n, s->ids.data(), s->mels.data(), s->rows.data(), s->valid.data(),
                                     s->keep.data(), s->decode ? nullptr : s->proj.data(), s->frames.data(),
                                     s->decode ? s->toks.data() : nullptr, s->decode ? s->ntok.data() : nullptr);
        if (st != UD_OK) return st;
        const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        for (int i = 0; i < n; ++i) s->recs[s->who[i]].idx = s->next[i];
        take_results(s, n, s->who.data(), s->keep.data(), seen.data(), s->toks.data(), s->ntok.data(), dt, &done);
        for (int i = 0; i < n; ++i) {
            StreamRec& r = s->recs[s->who[i]];
            if (!r.finished) trim_audio(s, r);
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

ud_status ud_streamer_emissions(ud_streamer* s, ud_streamer_id id, int32_t* tokens, int64_t* samples_seen,
                                double* compute_seconds, int cap, int* n) {
    StreamRec* r = rec_of(s, id);
    if (!r) return ud::host_fail(UD_ERR_NO_STREAM, "unknown streamer id");
    if (!n) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL count");
    const size_t k = r->tokens.size(), m = cap > 0 ? std::min(k, static_cast<size_t>(cap)) : 0;
    if (tokens && m) std::memcpy(tokens, r->tokens.data(), sizeof(int32_t) * m);
    if (samples_seen && m) std::memcpy(samples_seen, r->emit_samples.data(), sizeof(int64_t) * m);
    if (compute_seconds && m) std::memcpy(compute_seconds, r->emit_secs.data(), sizeof(double) * m);
    *n = static_cast<int>(k);
    return UD_OK;
}

ud_status ud_streamer_step_times(ud_streamer* s, ud_streamer_id id, double* out, int cap, int* n) {
    StreamRec* r = rec_of(s, id);
    if (!r) return ud::host_fail(UD_ERR_NO_STREAM, "unknown streamer id");
    if (!n) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL count");
    const size_t k = r->step_secs.size(), m = cap > 0 ? std::min(k, static_cast<size_t>(cap)) : 0;
    if (out && m) std::memcpy(out, r->step_secs.data(), sizeof(double) * m);
    *n = static_cast<int>(k);
    return UD_OK;
}

ud_status ud_streamer_release(ud_streamer* s, ud_streamer_id id) {
    StreamRec* r = rec_of(s, id);
    if (!r) return ud::host_fail(UD_ERR_NO_STREAM, "unknown streamer id");
    if (s->pend.active && std::find(s->pend.who.begin(), s->pend.who.end(), id) != s->pend.who.end()) {
        // the stream is in the step in flight: complete that step first; streams it finishes are reported by
        // the next ud_streamer_step
        ud_status st = ud_step_sync(s->e);
        if (st != UD_OK) return st;
        const size_t before = s->just_finished.size();
        int done = 0;
        take_pending(s, &done);
        s->carry.insert(s->carry.end(), s->just_finished.begin() + static_cast<std::ptrdiff_t>(before),
                        s->just_finished.end());
        s->just_finished.resize(before);
    }
    if (!r->finished && r->slot >= 0) ud_stream_close(s->e, r->slot);
    if (r->mel_id >= 0) ud_mel_stream_close(s->mel, r->mel_id);
    *r = StreamRec();
    s->free_ids.push_back(id);
    return UD_OK;
}

}  // extern "C"
