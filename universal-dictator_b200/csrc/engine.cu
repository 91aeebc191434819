// libud engine: the C ABI of include/ud.h over the sm_100a kernels.
//
// One engine = one CUDA device + one CUDA stream + shared weights + a pool of stream slots. It replaces
// MetalNemotronEncoder (Sources/DictatorEngine/Models/Nemotron.swift:51-91) and the per-stream
// FastConformerEncoder.StreamState (FastConformer.swift:406-435) with:
//   * paged per-stream K/V rings (pages of page_frames frames, kPageSlots page slots per stream, frame f at
//     row f % PF of page pages[(f / PF) % kPageSlots]); the roll is metadata only;
//   * a conv ring of conv_kernel-1 rows per (layer, stream);
//   * batched steps: the frames of all streams in a call are packed into one [M, d_model] activation block,
//     so every projection is one GEMM over M = sum of T (tcgen05 for bf16, FFMA for fp32).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "ud.h"

using namespace ud;

namespace {

thread_local std::string g_last_error;

ud_status fail(ud_status s, const std::string& msg) {
    g_last_error = msg;
    return s;
}

#define UD_CK(call)                                                                                  \
    do {                                                                                             \
        cudaError_t e_ = (call);                                                                     \
        if (e_ != cudaSuccess) return fail(UD_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

int nxt(int t) { return t / 2 + 1; }
int sub_len(int t) { return nxt(nxt(nxt(t))); }

struct WeightMat {
    void* p = nullptr;
    int N = 0, K = 0;
    TmaMatrix tma128, tma256;
    bool has_tma = false, has256 = false;
};

struct LayerW {
    WeightMat ff1_w1, ff1_w2, ff2_w1, ff2_w2, wqkv, wo, pw1, pw2;
    float *ln_ff1_g, *ln_ff1_b, *ln_att_g, *ln_att_b, *ln_conv_g, *ln_conv_b, *ln_cbn_g, *ln_cbn_b;
    float *ln_ff2_g, *ln_ff2_b, *ln_out_g, *ln_out_b;
    float *pos_u, *pos_v, *dw;
    void* ptab;
    TmaMatrix pmap;        // bf16 position table, boxes of 64 columns x 128 rows (the TMA attention kernel)
    bool has_pmap = false;
};

struct Slot {
    bool open = false;
    int lookahead = 0, step = 0, head = 0, cache_len = 0;
    int lp[kPageSlots];
    int pages[kPageSlots];
    void reset() {
        step = head = cache_len = 0;
        for (int i = 0; i < kPageSlots; ++i) lp[i] = pages[i] = -1;
    }
};

}  // namespace

struct ud_engine {
    ud_config cfg{};
    int device = 0;
    cudaStream_t stream = nullptr;
    // The layer stack of a batch of split_min_rows rows and up runs as two halves, the second on stream2, so that
    // one half's LayerNorm and tail CTAs share SMs with the other half's GEMMs: 2 % faster at 1024 streams x 14
    // frames, 3 % slower at 256 x 14 where the halves' GEMMs lose more to tile quantization (UD_SPLIT=<rows>,
    // 0: one stream). gstream is the stream the engine's GEMM dispatch enqueues on (null: `stream`).
    cudaStream_t stream2 = nullptr, gstream = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    int split_min_rows = 8192;
    int num_sms = 148;
    bool loaded = false;
    bool bf = true;
    int esz = 2;
    int tmax = 16, L = 70, D = 1024, H = 8, F = 4096, KC = 9, C = 256, F1 = 65, F2 = 33, F3 = 17, J = 640;
    int max_rows_in = 0;  // input rows per stream per step
    int in_width = 0;     // mel_bins or d_model
    int out_width = 0;    // joint_dim or d_model
    int Mcap = 0;
    std::vector<void*> allocs;
    std::vector<void*> host_allocs;

    std::vector<LayerW> layers;
    float *c0_w = nullptr, *c0_b = nullptr, *c2_w = nullptr, *c2_b = nullptr, *c5_w = nullptr, *c5_b = nullptr;
    float *c3_b = nullptr, *c6_b = nullptr, *out_b = nullptr;
    WeightMat c3, c6, sub_out, jenc;
    float* jenc_b = nullptr;
    RnntWeights rw{};
    RnntState rs{};
    RnntScratch rscr{};          // lock-step decoder scratch
    RnntTc rtc{};                // tensor-core decoder operands
    bool rnnt_lockstep = true;   // UD_RNNT_LOCKSTEP=0: one CTA per stream instead

    CacheGeom cg{};
    std::vector<int> free_pages;
    std::vector<Slot> slots;
    std::vector<int> free_slots;

    float* x = nullptr;
    void *h = nullptr, *hid = nullptr, *qkv = nullptr, *att = nullptr, *pw = nullptr, *y = nullptr;
    float* proj = nullptr;
    void *a2 = nullptr, *a3 = nullptr, *a4 = nullptr, *a5 = nullptr;
    float* subout = nullptr;
    float* in_stage = nullptr;
    float* out_stage = nullptr;
    int32_t* tok_dev = nullptr;
    int* ntok_dev = nullptr;
    void* gather_scratch = nullptr;

    float* h_in = nullptr;
    int* h_ntok = nullptr;

    // Pipelined host-buffer steps (ud_step_batch_async): staging buffer 1 and the copy streams (inputs, outputs:
    // separate, so step k+1's input copy does not queue behind step k's output copy), allocated on first use
    // (buffer 0 is in_stage / out_stage / tok_dev / ntok_dev / h_in). Step k uses buffer k % 2.
    cudaStream_t cstream = nullptr, ostream = nullptr;
    float *in_stage2 = nullptr, *out_stage2 = nullptr, *h_in2 = nullptr;
    int32_t* tok_dev2 = nullptr;
    int* ntok_dev2 = nullptr;
    int* err_async_h = nullptr;                                   // pinned [2]: device error flag after each step
    cudaEvent_t ev_in[2] = {}, ev_done[2] = {}, ev_out[2] = {};   // input copied, step computed, output copied
    int64_t async_issued = 0, async_completed = 0;

    static constexpr int kRing = 4;
    BatchEntry* meta_h[kRing] = {};
    BatchEntry* meta_d[kRing] = {};
    cudaEvent_t meta_ev[kRing] = {};
    int meta_i = 0;
    int* slots_h = nullptr;
    int* slots_d = nullptr;
    int* err_d = nullptr;
    int* err_h = nullptr;
    int64_t launches = 0;
    bool counted = false;   // included in the per-device engine count of the static decode scratch
    std::map<std::tuple<const void*, int, int, int>, TmaMatrix> amaps;
    std::map<std::tuple<const void*, int, int, int, int>, TmaMatrix> emaps;   // bf16 GEMM output blocks
    // CUDA graphs of the steady step, keyed by batch shape; metadata lives in a fixed device buffer for them
    struct GraphEntry {
        cudaGraphExec_t exec;
        int64_t kernels;
        std::vector<int> timer_kinds;   // kind of each timer slot its launches stamp (graph-mode timers on)
    };
    bool graphs_on = true;
    bool tc2_on = true;  // 2-CTA tcgen05 tiles for M >= 256, N % 256 == 0
    bool attn_tma_on = true;            // persistent TMA-fed attention (UD_ATTN_TMA=0: one CTA per stream-head)
    bool attn_maps = false;             // the tensor maps below exist
    TmaMatrix attn_qkv_map, attn_k_map, attn_v_map;   // QKV rows (64 x 16 boxes), K and V page pools
    BatchEntry* meta_graph_d = nullptr;
    // key: n, rows_max, M, tmax_b, tokens, staging buffer, the halves' split row, graph-mode timers
    std::map<std::tuple<int, int, int, int, int, int, int, int>, GraphEntry> graphs;
    std::map<std::tuple<int, int, int, int, int, int, int, int>, int> graph_seen;
    // graph-mode kernel timers: [kTimerSlots] first-start times, then [kTimerSlots] last-finish times (ns)
    bool timers = false;
    unsigned long long* timer_buf = nullptr;
    std::vector<int> timer_kinds;        // kind of each slot handed out while the current step is enqueued
    std::vector<int> timer_last_kinds;   // the slots of the last step run
    // per-kernel-class timing
    bool prof = false;
    std::vector<cudaEvent_t> prof_events;
    std::vector<std::pair<int, size_t>> prof_marks;  // (kind, index of the begin event; end = index + 1)
    size_t prof_used = 0;
    double prof_ms[UD_KIND_COUNT] = {};
    int64_t prof_n[UD_KIND_COUNT] = {};
};

namespace {

// Counts one launch of this library's kernels and, when profiling, brackets it with events.
struct Launch {
    ud_engine* e;
    int kind;
    size_t idx = 0;
    bool on;
    Launch(ud_engine* e_, int k) : e(e_), kind(k), on(e_->prof) {
        if (!on) return;
        if (e->prof_used + 2 > e->prof_events.size()) {
            for (int i = 0; i < 256; ++i) {
                cudaEvent_t ev;
                cudaEventCreate(&ev);
                e->prof_events.push_back(ev);
            }
        }
        idx = e->prof_used;
        e->prof_used += 2;
        cudaEventRecord(e->prof_events[idx], e->stream);
    }
    ~Launch() {
        e->launches++;
        if (!on) return;
        cudaEventRecord(e->prof_events[idx + 1], e->stream);
        e->prof_marks.emplace_back(kind, idx);
    }
};

void prof_flush(ud_engine* e) {
    if (e->prof_marks.empty()) return;
    cudaStreamSynchronize(e->stream);
    for (auto& m : e->prof_marks) {
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, e->prof_events[m.second], e->prof_events[m.second + 1]) == cudaSuccess) {
            e->prof_ms[m.first] += ms;
            e->prof_n[m.first] += 1;
        }
    }
    cudaGetLastError();
    e->prof_marks.clear();
    e->prof_used = 0;
}

template <typename T>
ud_status dalloc(ud_engine* e, T** p, size_t count) {
    void* q = nullptr;
    if (count == 0) count = 1;
    if (cudaMalloc(&q, count * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return fail(UD_ERR_OUT_OF_MEMORY, "cudaMalloc of " + std::to_string(count * sizeof(T)) + " bytes failed");
    }
    e->allocs.push_back(q);
    *p = static_cast<T*>(q);
    return UD_OK;
}

ud_status dalloc_bytes(ud_engine* e, void** p, size_t bytes) {
    return dalloc<uint8_t>(e, reinterpret_cast<uint8_t**>(p), bytes);
}

template <typename T>
ud_status halloc(ud_engine* e, T** p, size_t count) {
    void* q = nullptr;
    if (count == 0) count = 1;
    if (cudaMallocHost(&q, count * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return fail(UD_ERR_OUT_OF_MEMORY, "cudaMallocHost failed");
    }
    e->host_allocs.push_back(q);
    *p = static_cast<T*>(q);
    return UD_OK;
}

#define UD_TRY(x)                      \
    do {                               \
        ud_status s_ = (x);            \
        if (s_ != UD_OK) return s_;    \
    } while (0)

bool tc_ok(int N, int K) { return N % 128 == 0 && K % 64 == 0; }

// Cached tensor maps: a bf16 activation operand [M, K] (128-row boxes), and a GEMM output [M, N] in 32-row blocks
// for the TMA epilogues (null when a map cannot describe it).
const TmaMatrix* act_map(ud_engine* e, const void* A, int M, int K, int lda) {
    auto key = std::make_tuple(A, M, K, lda);
    auto it = e->amaps.find(key);
    if (it == e->amaps.end()) {
        TmaMatrix t;
        if (!make_tma_bf16(t, A, M, K, lda, 128)) return nullptr;
        it = e->amaps.emplace(key, t).first;
    }
    return &it->second;
}
const TmaMatrix* out_map(ud_engine* e, const void* p, int M, int N, int ld, bool bf) {
    const auto k = std::make_tuple(p, M, N, ld, bf ? 1 : 0);
    auto jt = e->emaps.find(k);
    if (jt == e->emaps.end()) {
        TmaMatrix t;
        if (!make_tma_epi(t, p, M, N, ld, bf)) return nullptr;
        jt = e->emaps.emplace(k, t).first;
    }
    return &jt->second;
}

// One GEMM through the engine's dispatch: tcgen05 for bf16 with more than 16 rows, SIMT otherwise.
// A graph-mode timer slot for the next launch of this kind, or null (timers off, or every slot handed out).
unsigned long long* timer_slot(ud_engine* e, int kind) {
    if (!e->timers || static_cast<int>(e->timer_kinds.size()) >= kTimerSlots) return nullptr;
    e->timer_kinds.push_back(kind);
    return e->timer_buf + (e->timer_kinds.size() - 1);
}

ud_status gemm(ud_engine* e, const void* A, int lda, int M, const WeightMat& W, const GemmEpilogue& epi) {
    if (M <= 0) return UD_OK;
    cudaStream_t const gs = e->gstream ? e->gstream : e->stream;
    const bool tc = e->bf && M > 16 && W.has_tma;
    const bool tc2 = tc && e->tc2_on && M >= 256 && W.N % 16 == 0;
    Launch L_(e, tc2 ? UD_KIND_GEMM_TC2 : tc ? UD_KIND_GEMM_TC : UD_KIND_GEMM_SIMT);
    GemmEpilogue ep = epi;
    if (tc2) ep.prof = timer_slot(e, UD_KIND_GEMM_TC2);
    if (e->bf) {
        if (!tc) {
            gemm_simt<bf16, bf16>(static_cast<const bf16*>(A), lda, static_cast<const bf16*>(W.p), M, W.N, W.K, epi,
                                  gs);
        } else {
            const TmaMatrix* am = act_map(e, A, M, W.K, lda);
            if (!am) return fail(UD_ERR_CUDA, "cuTensorMapEncodeTiled failed for an activation operand");
            if (tc2) {
                // output maps for the TMA epilogues: bf16 stores, and fp32 reduce-adds when the residual is the output
                const TmaMatrix* om = nullptr;
                if (epi.out_bf16 && !epi.residual)
                    om = out_map(e, epi.out, M, W.N, epi.ldo, true);
                else if (!epi.out_bf16 && epi.residual == epi.out && epi.ldr == epi.ldo && epi.res_scale == 1.f)
                    om = out_map(e, epi.out, M, W.N, epi.ldo, false);
                gemm_tc2(*am, W.tma128, M, W.N, W.K, 256, ep, e->err_d, e->num_sms, om, gs);
            } else {
                const int bn = W.has256 ? gemm_tc_pick_bn(M, W.N, e->num_sms) : 128;
                gemm_tc(*am, bn == 256 ? W.tma256 : W.tma128, M, W.N, W.K, bn, epi, e->err_d, e->num_sms, gs);
            }
        }
    } else {
        gemm_simt<float, float>(static_cast<const float*>(A), lda, static_cast<const float*>(W.p), M, W.N, W.K, epi,
                                gs);
    }
    return UD_OK;
}

GemmEpilogue epi_out(void* out, int ldo, bool out_act_dtype, const ud_engine* e) {
    GemmEpilogue g;
    g.out = out;
    g.ldo = ldo;
    g.out_bf16 = (out_act_dtype && e->bf) ? 1 : 0;
    return g;
}

// The status of a nonzero device error flag value; clears the flag.
ud_status device_error_status(ud_engine* e, int code) {
    UD_CK(cudaMemsetAsync(e->err_d, 0, sizeof(int), e->stream));
    UD_CK(cudaStreamSynchronize(e->stream));
    static const char* names[] = {"ok", "GEMM TMA stage wait", "GEMM free-stage wait", "GEMM accumulator wait",
                                  "GEMM TMEM drain wait", "unmapped cache page", "test wait",
                                  "RNN-T grid barrier wait", "attention stage wait",
                                  "RNN-T decoder input beyond the fp16 range", "conv module copy wait",
                                  "cache gather copy wait"};
    const char* nm = (code >= 0 && code <= 11) ? names[code] : "unknown";
    if (code == DEV_BAD_PAGE || code == DEV_RANGE_F16)
        return fail(UD_ERR_INVALID_ARGUMENT, std::string("device reported: ") + nm);
    return fail(UD_ERR_DEVICE_TIMEOUT, std::string("device wait expired: ") + nm);
}

ud_status check_device_error(ud_engine* e) {
    UD_CK(cudaMemcpyAsync(e->err_h, e->err_d, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    UD_CK(cudaStreamSynchronize(e->stream));
    const int code = *e->err_h;
    return code != 0 ? device_error_status(e, code) : UD_OK;
}

// Completes every outstanding pipelined step (output copies done); the first device error among them is the
// status.
ud_status drain_async(ud_engine* e) {
    if (!e->cstream || e->async_completed == e->async_issued) return UD_OK;
    UD_CK(cudaStreamSynchronize(e->cstream));
    UD_CK(cudaStreamSynchronize(e->ostream));
    int code = 0;
    for (; e->async_completed < e->async_issued; ++e->async_completed) {
        const int b = static_cast<int>(e->async_completed & 1);
        if (code == 0) code = e->err_async_h[b];
    }
    return code != 0 ? device_error_status(e, code) : UD_OK;
}

// Staging buffer 1, the copy stream and the events of the pipelined steps, on first use.
ud_status async_setup(ud_engine* e) {
    if (e->cstream) return UD_OK;
    const size_t B = static_cast<size_t>(e->cfg.max_batch);
    const size_t in_elems = B * e->max_rows_in * e->in_width;
    const size_t out_elems = B * e->tmax * e->out_width;
    const size_t tok_elems = B * e->tmax * e->cfg.max_symbols;
    UD_TRY(dalloc(e, &e->in_stage2, in_elems));
    UD_TRY(dalloc(e, &e->out_stage2, out_elems));
    UD_TRY(dalloc(e, &e->tok_dev2, tok_elems));
    UD_TRY(dalloc(e, &e->ntok_dev2, B));
    UD_TRY(halloc(e, &e->h_in2, in_elems));
    UD_TRY(halloc(e, &e->err_async_h, 2));
    e->err_async_h[0] = e->err_async_h[1] = 0;
    for (int b = 0; b < 2; ++b)
        for (cudaEvent_t* ev : {&e->ev_in[b], &e->ev_done[b], &e->ev_out[b]})
            if (!*ev) UD_CK(cudaEventCreateWithFlags(ev, cudaEventDisableTiming));
    UD_CK(cudaStreamCreateWithFlags(&e->ostream, cudaStreamNonBlocking));
    UD_CK(cudaStreamCreateWithFlags(&e->cstream, cudaStreamNonBlocking));
    return UD_OK;
}

// ---------------------------------------------------------------- pages
void free_out_of_window(ud_engine* e, Slot& s) {
    const int PF = e->cfg.page_frames;
    const int win_lo = s.head - e->L;  // first frame still in the left context
    for (int i = 0; i < kPageSlots; ++i) {
        if (s.lp[i] >= 0 && (s.lp[i] + 1) * PF <= win_lo) {
            e->free_pages.push_back(s.pages[i]);
            s.lp[i] = s.pages[i] = -1;
        }
    }
}

void free_all_pages(ud_engine* e, Slot& s) {
    for (int i = 0; i < kPageSlots; ++i) {
        if (s.lp[i] >= 0) e->free_pages.push_back(s.pages[i]);
        s.lp[i] = s.pages[i] = -1;
    }
}

// Maps pages for frames [s.head, s.head + k). Records what it mapped so a failed batch can undo it.
ud_status map_pages(ud_engine* e, Slot& s, int k, std::vector<std::pair<Slot*, int>>& undo) {
    const int PF = e->cfg.page_frames;
    for (int f = s.head; f < s.head + k; ++f) {
        const int lp = f / PF, ps = lp % kPageSlots;
        if (s.lp[ps] == lp) continue;
        if (s.lp[ps] >= 0)
            return fail(UD_ERR_INVALID_ARGUMENT, "page ring overflow: a chunk plus the left context exceeds the ring");
        if (e->free_pages.empty()) return fail(UD_ERR_POOL_EXHAUSTED, "cache page pool exhausted");
        s.pages[ps] = e->free_pages.back();
        e->free_pages.pop_back();
        s.lp[ps] = lp;
        undo.emplace_back(&s, ps);
    }
    return UD_OK;
}

void undo_pages(ud_engine* e, std::vector<std::pair<Slot*, int>>& undo) {
    for (auto it = undo.rbegin(); it != undo.rend(); ++it) {
        e->free_pages.push_back(it->first->pages[it->second]);
        it->first->lp[it->second] = it->first->pages[it->second] = -1;
    }
    undo.clear();
}

BatchEntry* next_meta_host(ud_engine* e, int* ring_index) {
    const int mi = e->meta_i;
    cudaEventSynchronize(e->meta_ev[mi]);
    *ring_index = mi;
    return e->meta_h[mi];
}

ud_status upload_meta(ud_engine* e, int mi, int n) {
    UD_CK(cudaMemcpyAsync(e->meta_d[mi], e->meta_h[mi], sizeof(BatchEntry) * n, cudaMemcpyHostToDevice, e->stream));
    UD_CK(cudaEventRecord(e->meta_ev[mi], e->stream));
    e->meta_i = (mi + 1) % ud_engine::kRing;
    return UD_OK;
}

ud_status check_ids(ud_engine* e, int n, const ud_stream_id* ids) {
    if (n < 1 || n > e->cfg.max_batch) return fail(UD_ERR_INVALID_ARGUMENT, "batch size out of range");
    if (!ids) return fail(UD_ERR_INVALID_ARGUMENT, "ids is NULL");
    std::vector<int> seen;
    seen.reserve(n);
    for (int i = 0; i < n; ++i) {
        const int id = ids[i];
        if (id < 0 || id >= e->cfg.max_streams || !e->slots[id].open)
            return fail(UD_ERR_NO_STREAM, "unknown or closed stream id " + std::to_string(id));
        seen.push_back(id);
    }
    std::sort(seen.begin(), seen.end());
    if (std::adjacent_find(seen.begin(), seen.end()) != seen.end())
        return fail(UD_ERR_INVALID_ARGUMENT, "a stream id appears twice in one batch");
    return UD_OK;
}

// ---------------------------------------------------------------- the batched step
// Enqueues every kernel of one batched step on the engine stream (also the body of a captured graph).
// One step of n streams (metadata md, M rows) on the engine stream. With 0 < n_a < n the layer stack runs as two
// halves: streams [0, n_a) (rows [0, m_a)) on the engine stream, the rest on stream2.
ud_status enqueue_step(ud_engine* e, const BatchEntry* md, int n, int M, int tmax_b, int rows_max, const float* in_dev,
                       int rows_stride, float* out_dev, int32_t* tokens_dev, int* ntok_dev, int n_a, int m_a) {
    const bool sub = e->cfg.sub_channels > 0;
    const int D = e->D;
    cudaStream_t st = e->stream;
    // ---- encoder input: subsampling, or frames as given
    if (sub) {
        const int Tin = rows_max, T1 = nxt(Tin), T2 = nxt(T1), T3 = nxt(T2), C = e->C;
        {
            Launch L_(e, UD_KIND_SUBSAMPLE);
            if (e->bf)
                sub_conv01<bf16>(in_dev, rows_stride, e->cfg.mel_bins, md, n, Tin, e->c0_w, e->c0_b, T1, e->F1, e->c2_w,
                                 e->c2_b, (bf16*)e->a2, T2, e->F2, C, e->num_sms, st);
            else
                sub_conv01<float>(in_dev, rows_stride, e->cfg.mel_bins, md, n, Tin, e->c0_w, e->c0_b, T1, e->F1, e->c2_w,
                                  e->c2_b, (float*)e->a2, T2, e->F2, C, e->num_sms, st);
        }
        GemmEpilogue g3 = epi_out(e->a3, C, true, e);
        g3.bias = e->c3_b;
        g3.act = ACT_RELU;
        UD_TRY(gemm(e, e->a2, C, n * T2 * e->F2, e->c3, g3));
        {
        Launch L_(e, UD_KIND_SUBSAMPLE);
        if (e->bf)
            sub_dwconv2<bf16>((bf16*)e->a3, T2, e->F2, md, n, e->c5_w, e->c5_b, (bf16*)e->a4, T3, e->F3, C, st);
        else
            sub_dwconv2<float>((float*)e->a3, T2, e->F2, md, n, e->c5_w, e->c5_b, (float*)e->a4, T3, e->F3, C, st);
        }
        GemmEpilogue g6 = epi_out(e->a5, C, true, e);
        g6.bias = e->c6_b;
        g6.act = ACT_RELU;
        UD_TRY(gemm(e, e->a4, C, n * T3 * e->F3, e->c6, g6));
        GemmEpilogue go = epi_out(e->subout, D, false, e);
        go.bias = e->out_b;
        UD_TRY(gemm(e, e->a5, e->F3 * C, n * T3, e->sub_out, go));
        {
            Launch L_(e, UD_KIND_SUBSAMPLE);
            sub_select<float>(e->subout, T3, e->out_b, md, n, e->x, D, st);
        }
    } else {
        Launch L_(e, UD_KIND_SUBSAMPLE);
        pack_frames(in_dev, rows_stride, md, n, tmax_b, e->x, D, st);
    }

    // ---- conformer layers, over the streams md[0, nh) whose rows are [row0, row0 + Mh), on stream sh. The row
    // kernels (LayerNorm, GEMMs) take the half's rows; the per-stream kernels (attention, conv module) take the
    // half's metadata, whose row offsets index the whole batch's buffers.
    const int NL = e->cfg.n_layers;
    auto run_layers = [&](const BatchEntry* mdh, int nh, int row0, int Mh, cudaStream_t sh) -> ud_status {
        e->gstream = sh;
        const size_t es = e->esz;
        float* x = e->x + static_cast<size_t>(row0) * D;
        void* h = static_cast<char*>(e->h) + static_cast<size_t>(row0) * D * es;
        void* hid = static_cast<char*>(e->hid) + static_cast<size_t>(row0) * e->F * es;
        void* qkv = static_cast<char*>(e->qkv) + static_cast<size_t>(row0) * 3 * D * es;
        void* att = static_cast<char*>(e->att) + static_cast<size_t>(row0) * D * es;
        void* pw = static_cast<char*>(e->pw) + static_cast<size_t>(row0) * 2 * D * es;
        void* y = static_cast<char*>(e->y) + static_cast<size_t>(row0) * D * es;
        auto ln = [&](const float* g, const float* b) {
            Launch L_(e, UD_KIND_NORM);
            if (e->bf) layer_norm<bf16>(x, g, b, (bf16*)h, Mh, D, sh, timer_slot(e, UD_KIND_NORM));
            else layer_norm<float>(x, g, b, (float*)h, Mh, D, sh, timer_slot(e, UD_KIND_NORM));
        };
        auto resid = [&](float scale) {
            GemmEpilogue g = epi_out(x, D, false, e);
            g.residual = x;
            g.ldr = D;
            g.out_scale = scale;
            return g;
        };
        // A feed-forward module: x += 1/2 * (SiLU(h W1^T) W2^T).
        auto ff = [&](const WeightMat& w1, const WeightMat& w2) -> ud_status {
            GemmEpilogue gs = epi_out(hid, e->F, true, e);
            gs.act = ACT_SILU;
            UD_TRY(gemm(e, h, D, Mh, w1, gs));
            return gemm(e, hid, e->F, Mh, w2, resid(0.5f));
        };
        if (NL > 0) ln(e->layers[0].ln_ff1_g, e->layers[0].ln_ff1_b);
        for (int l = 0; l < NL; ++l) {
            LayerW& w = e->layers[l];
            UD_TRY(ff(w.ff1_w1, w.ff1_w2));
            ln(w.ln_att_g, w.ln_att_b);
            UD_TRY(gemm(e, h, D, Mh, w.wqkv, epi_out(qkv, 3 * D, true, e)));
            {
            Launch L_(e, UD_KIND_ATTENTION);
            const bool tma_done = e->bf && e->attn_tma_on && e->attn_maps && w.has_pmap &&
                                  relpos_attention_tma(e->attn_qkv_map, e->attn_k_map, e->attn_v_map, w.pmap,
                                                       e->tmax - 16, w.pos_u, w.pos_v, mdh, nh, tmax_b, e->cg, l,
                                                       (bf16*)e->att, D, e->H, e->num_sms, e->err_d, sh,
                                                       timer_slot(e, UD_KIND_ATTENTION));
            if (tma_done) {
            } else if (e->bf)
                relpos_attention<bf16>((bf16*)e->qkv, 3 * D, (bf16*)w.ptab, e->tmax, w.pos_u, w.pos_v, mdh, nh, tmax_b,
                                       e->cg, l, (bf16*)e->att, D, e->H, e->err_d, sh);
            else
                relpos_attention<float>((float*)e->qkv, 3 * D, (float*)w.ptab, e->tmax, w.pos_u, w.pos_v, mdh, nh,
                                        tmax_b, e->cg, l, (float*)e->att, D, e->H, e->err_d, sh);
            }
            UD_TRY(gemm(e, att, D, Mh, w.wo, resid(1.0f)));
            ln(w.ln_conv_g, w.ln_conv_b);
            UD_TRY(gemm(e, h, D, Mh, w.pw1, epi_out(pw, 2 * D, true, e)));
            {
            Launch L_(e, UD_KIND_CONV);
            if (e->bf)
                conv_module<bf16>((bf16*)e->pw, 2 * D, w.dw, w.ln_cbn_g, w.ln_cbn_b, mdh, nh, tmax_b, e->cg, l, e->KC,
                                  (bf16*)e->y, D, e->err_d, sh, timer_slot(e, UD_KIND_CONV));
            else
                conv_module<float>((float*)e->pw, 2 * D, w.dw, w.ln_cbn_g, w.ln_cbn_b, mdh, nh, tmax_b, e->cg, l, e->KC,
                                   (float*)e->y, D, e->err_d, sh, timer_slot(e, UD_KIND_CONV));
            }
            UD_TRY(gemm(e, y, D, Mh, w.pw2, resid(1.0f)));
            ln(w.ln_ff2_g, w.ln_ff2_b);
            UD_TRY(ff(w.ff2_w1, w.ff2_w2));
            if (l + 1 < NL) {
                LayerW& nx = e->layers[l + 1];
                Launch L_(e, UD_KIND_NORM);
                if (e->bf)
                    layer_norm2<bf16>(x, w.ln_out_g, w.ln_out_b, nx.ln_ff1_g, nx.ln_ff1_b, (bf16*)h, Mh, D, sh,
                                      timer_slot(e, UD_KIND_NORM));
                else
                    layer_norm2<float>(x, w.ln_out_g, w.ln_out_b, nx.ln_ff1_g, nx.ln_ff1_b, (float*)h, Mh, D, sh,
                                       timer_slot(e, UD_KIND_NORM));
            } else if (e->cfg.joint_dim) {
                ln(w.ln_out_g, w.ln_out_b);  // h = LN_out(x): the joint's operand
            } else {
                Launch L_(e, UD_KIND_NORM);
                layer_norm<float>(x, w.ln_out_g, w.ln_out_b, x, Mh, D, sh, timer_slot(e, UD_KIND_NORM));
            }
        }
        return UD_OK;
    };
    if (n_a > 0 && n_a < n && NL > 0) {
        // two halves: fork stream2 from the step's stream, join it back before the joint projection
        UD_CK(cudaEventRecord(e->ev_fork, st));
        UD_CK(cudaStreamWaitEvent(e->stream2, e->ev_fork, 0));
        ud_status sa = run_layers(md, n_a, 0, m_a, st);
        ud_status sb = sa == UD_OK ? run_layers(md + n_a, n - n_a, m_a, M - m_a, e->stream2) : sa;
        e->gstream = nullptr;
        UD_CK(cudaEventRecord(e->ev_join, e->stream2));   // joined even after an error, so a capture can end
        UD_CK(cudaStreamWaitEvent(st, e->ev_join, 0));
        UD_TRY(sb);
    } else {
        const ud_status sa = run_layers(md, n, 0, M, st);
        e->gstream = nullptr;
        UD_TRY(sa);
    }

    // ---- joint encoder projection, outputs, RNN-T
    if (e->cfg.joint_dim) {
        GemmEpilogue gj = epi_out(e->proj, e->J, false, e);
        gj.bias = e->jenc_b;
        UD_TRY(gemm(e, e->h, D, M, e->jenc, gj));
        {
            Launch L_(e, UD_KIND_OTHER);
            scatter_rows(e->proj, md, n, out_dev, e->tmax, e->J, st);
        }
        if (tokens_dev) {
            Launch L_(e, UD_KIND_RNNT);
            rnnt_greedy(e->rw, e->rs, e->proj, e->J, md, n, tokens_dev, e->tmax * e->cfg.max_symbols, ntok_dev,
                        e->rnnt_lockstep ? &e->rscr : nullptr, e->num_sms, e->err_d, st);
        }
    } else {
        Launch L_(e, UD_KIND_OTHER);
        scatter_rows(e->x, md, n, out_dev, e->tmax, D, st);
    }
    return UD_OK;
}

ud_status run_batch(ud_engine* e, int n, const ud_stream_id* ids, const float* in_dev, int rows_stride,
                    const int* n_rows, const int* valid_rows, const int* keep_all, float* out_dev, int* frames_out,
                    int32_t* tokens_dev, int* ntok_dev, bool graph_ok) {
    if (!e->loaded) return fail(UD_ERR_NOT_READY, "weights not loaded");
    UD_TRY(check_ids(e, n, ids));
    if (!n_rows || !valid_rows || !in_dev || !out_dev) return fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (tokens_dev && !e->cfg.joint_dim) return fail(UD_ERR_INVALID_ARGUMENT, "no RNN-T head in this configuration");
    const bool sub = e->cfg.sub_channels > 0;
    const int L = e->L, D = e->D;
    int mi = 0;
    BatchEntry* mh = next_meta_host(e, &mi);
    int M = 0, tmax_b = 0, rows_max = 0;
    for (int i = 0; i < n; ++i) {
        Slot& s = e->slots[ids[i]];
        const int nr = n_rows[i], vr = valid_rows[i];
        if (nr < 1 || nr > rows_stride || nr > e->max_rows_in || vr < 0 || vr > nr)
            return fail(UD_ERR_INVALID_ARGUMENT, "n_rows/valid_rows out of range for stream " + std::to_string(ids[i]));
        int drop = 0, T, vt, keep;
        if (sub) {
            drop = s.step == 0 ? 0 : 2;
            T = sub_len(nr) - drop;
            vt = std::max(0, std::min(sub_len(vr) - drop, T));
            keep = (keep_all && keep_all[i]) ? vt : std::min(vt, s.lookahead + 1);
        } else {
            T = nr;
            vt = vr;
            keep = T;
        }
        if (T < 1 || T > e->tmax)
            return fail(UD_ERR_INVALID_ARGUMENT, "chunk of " + std::to_string(T) + " frames outside [1, max_chunk_frames]");
        BatchEntry& b = mh[i];
        b.slot = ids[i];
        b.row_off = M;
        b.T = T;
        b.valid_t = vt;
        b.cache_len = s.cache_len;
        b.head = s.head;
        b.drop = drop;
        b.valid_mel = vr;
        b.n_rows = nr;
        b.keep = keep;
        b.tok_off = i * e->tmax * e->cfg.max_symbols;
        b.pad = 0;
        M += T;
        tmax_b = std::max(tmax_b, T);
        rows_max = std::max(rows_max, nr);
    }
    std::vector<std::pair<Slot*, int>> undo;
    for (int i = 0; i < n; ++i) {
        ud_status st = map_pages(e, e->slots[ids[i]], mh[i].T, undo);
        if (st != UD_OK) {
            undo_pages(e, undo);
            return st;
        }
        std::memcpy(mh[i].pages, e->slots[ids[i]].pages, sizeof(mh[i].pages));
    }
    // Two halves for the layer stack of a large batch, each with enough rows for the 2-CTA GEMM tiles (not while
    // profiling: per-kind times are taken on one stream).
    int n_a = 0, m_a = 0;
    if (e->split_min_rows > 0 && !e->prof && n >= 2 && M >= std::max(1024, e->split_min_rows)) {
        n_a = n / 2;
        m_a = mh[n_a].row_off;
        if (m_a < 512 || M - m_a < 512) n_a = m_a = 0;
    }
    const std::tuple<int, int, int, int, int, int, int, int> key{n, rows_max, M, tmax_b, tokens_dev ? 1 : 0,
                                                                 in_dev == e->in_stage ? 0 : 1, m_a,
                                                                 e->timers ? 1 : 0};
    const bool use_graph = graph_ok && e->graphs_on && !e->prof;
    if (e->timers) {   // every slot empty: starts at the largest value, finishes at zero
        UD_CK(cudaMemsetAsync(e->timer_buf, 0xff, sizeof(unsigned long long) * kTimerSlots, e->stream));
        UD_CK(cudaMemsetAsync(e->timer_buf + kTimerSlots, 0, sizeof(unsigned long long) * kTimerSlots, e->stream));
    }
    e->timer_kinds.clear();
    if (!use_graph) {
        UD_TRY(upload_meta(e, mi, n));
        UD_TRY(enqueue_step(e, e->meta_d[mi], n, M, tmax_b, rows_max, in_dev, rows_stride, out_dev, tokens_dev, ntok_dev,
                            n_a, m_a));
        e->timer_last_kinds = e->timer_kinds;
    } else {
        // Metadata for the graph's fixed buffer; the pinned source slot is protected by the ring's event.
        UD_CK(cudaMemcpyAsync(e->meta_graph_d, mh, sizeof(BatchEntry) * n, cudaMemcpyHostToDevice, e->stream));
        UD_CK(cudaEventRecord(e->meta_ev[mi], e->stream));
        e->meta_i = (mi + 1) % ud_engine::kRing;
        auto it = e->graphs.find(key);
        if (it == e->graphs.end() && e->graph_seen[key] >= 1) {
            if (e->graphs.size() >= 16) {
                for (auto& g : e->graphs) cudaGraphExecDestroy(g.second.exec);
                e->graphs.clear();
            }
            const int64_t before = e->launches;
            UD_CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
            const ud_status cs = enqueue_step(e, e->meta_graph_d, n, M, tmax_b, rows_max, in_dev, rows_stride, out_dev,
                                              tokens_dev, ntok_dev, n_a, m_a);
            cudaGraph_t graph = nullptr;
            const cudaError_t ce = cudaStreamEndCapture(e->stream, &graph);
            const int64_t kernels = e->launches - before;
            e->launches = before;
            if (cs != UD_OK || ce != cudaSuccess) {
                if (graph) cudaGraphDestroy(graph);
                cudaGetLastError();
                return cs != UD_OK ? cs : fail(UD_ERR_CUDA, std::string("stream capture failed: ") + cudaGetErrorString(ce));
            }
            cudaGraphExec_t exec = nullptr;
            const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
            cudaGraphDestroy(graph);
            if (ie != cudaSuccess) return fail(UD_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(ie));
            it = e->graphs.emplace(key, ud_engine::GraphEntry{exec, kernels, e->timer_kinds}).first;
        }
        if (it != e->graphs.end()) {
            UD_CK(cudaGraphLaunch(it->second.exec, e->stream));
            e->launches += it->second.kernels;
            e->timer_last_kinds = it->second.timer_kinds;
        } else {
            e->graph_seen[key] += 1;
            e->timer_kinds.clear();
            UD_TRY(enqueue_step(e, e->meta_graph_d, n, M, tmax_b, rows_max, in_dev, rows_stride, out_dev, tokens_dev,
                                ntok_dev, n_a, m_a));
            e->timer_last_kinds = e->timer_kinds;
        }
    }
    UD_CK(cudaGetLastError());

    // ---- roll: metadata only
    for (int i = 0; i < n; ++i) {
        Slot& s = e->slots[ids[i]];
        s.head += mh[i].T;
        s.cache_len = std::min(s.cache_len + mh[i].T, L);
        s.step += 1;
        free_out_of_window(e, s);
        if (frames_out) frames_out[i] = mh[i].keep;
    }
    return UD_OK;
}

// ---------------------------------------------------------------- weights
struct WeightTable {
    std::map<std::string, const ud_weight*> by_name;
};

ud_status need(const WeightTable& t, const std::string& name, std::vector<int64_t> shape, const float** out) {
    auto it = t.by_name.find(name);
    if (it == t.by_name.end()) return fail(UD_ERR_WEIGHTS, "missing weight " + name);
    const ud_weight* w = it->second;
    bool ok = w->ndim == static_cast<int>(shape.size()) && w->data;
    for (size_t i = 0; ok && i < shape.size(); ++i) ok = w->shape[i] == shape[i];
    if (!ok) return fail(UD_ERR_WEIGHTS, "weight " + name + " has the wrong shape");
    *out = w->data;
    return UD_OK;
}

ud_status upload_f32(ud_engine* e, const float* host, size_t n, float** out) {
    UD_TRY(dalloc(e, out, n));
    UD_CK(cudaMemcpyAsync(*out, host, n * sizeof(float), cudaMemcpyHostToDevice, e->stream));
    return UD_OK;
}

// Device fp32 staging for conversions (largest single weight).
struct Staging {
    float* p = nullptr;
    size_t cap = 0;
};

ud_status upload_gemm(ud_engine* e, Staging& stg, const std::vector<const float*>& parts, const std::vector<int>& part_rows,
                      int K, WeightMat& W) {
    int N = 0;
    for (int r : part_rows) N += r;
    W.N = N;
    W.K = K;
    const size_t n = static_cast<size_t>(N) * K;
    if (e->bf) {
        if (n > stg.cap) return fail(UD_ERR_WEIGHTS, "staging buffer too small");
        size_t off = 0;
        for (size_t i = 0; i < parts.size(); ++i) {
            UD_CK(cudaMemcpyAsync(stg.p + off, parts[i], sizeof(float) * part_rows[i] * K, cudaMemcpyHostToDevice,
                                  e->stream));
            off += static_cast<size_t>(part_rows[i]) * K;
        }
        void* p;
        UD_TRY(dalloc_bytes(e, &p, n * 2));
        f32_to_bf16(stg.p, static_cast<bf16*>(p), n, e->stream);
        UD_CK(cudaStreamSynchronize(e->stream));
        W.p = p;
        if (tc_ok(N, K)) {
            if (!make_tma_bf16(W.tma128, p, N, K, K, 128)) return fail(UD_ERR_CUDA, "tensor map for a weight failed");
            W.has_tma = true;
            if (N % 256 == 0) {
                if (!make_tma_bf16(W.tma256, p, N, K, K, 256)) return fail(UD_ERR_CUDA, "tensor map for a weight failed");
                W.has256 = true;
            }
        }
    } else {
        float* p;
        UD_TRY(dalloc(e, &p, n));
        size_t off = 0;
        for (size_t i = 0; i < parts.size(); ++i) {
            UD_CK(cudaMemcpyAsync(p + off, parts[i], sizeof(float) * part_rows[i] * K, cudaMemcpyHostToDevice, e->stream));
            off += static_cast<size_t>(part_rows[i]) * K;
        }
        W.p = p;
    }
    return UD_OK;
}

// NeMo RelPositionalEncoding rows (fp32 as torch computes them) for rel in [lo, hi].
std::vector<float> sinusoid_rows(int lo, int hi, int D) {
    std::vector<float> pe(static_cast<size_t>(hi - lo + 1) * D);
    const float k = static_cast<float>(-(std::log(10000.0) / D));
    for (int r = lo; r <= hi; ++r) {
        float* row = &pe[static_cast<size_t>(r - lo) * D];
        for (int i = 0; i < D; i += 2) {
            const float div = std::exp(static_cast<float>(i) * k);
            const float ang = static_cast<float>(r) * div;
            row[i] = std::sin(ang);
            row[i + 1] = std::cos(ang);
        }
    }
    return pe;
}

ud_status load_weights_impl(ud_engine* e, const ud_weight* table, int n) {
    WeightTable t;
    for (int i = 0; i < n; ++i) {
        if (!table[i].name) return fail(UD_ERR_WEIGHTS, "weight without a name");
        t.by_name[table[i].name] = &table[i];
    }
    const ud_config& c = e->cfg;
    const int D = e->D, F = e->F, H = e->H, DK = D / H, C = e->C, L = e->L;
    Staging stg;
    stg.cap = std::max<size_t>({static_cast<size_t>(3) * D * D, static_cast<size_t>(F) * D,
                                static_cast<size_t>(D) * C * e->F3, static_cast<size_t>(2) * D * D});
    UD_TRY(dalloc(e, &stg.p, stg.cap));
    const float* p = nullptr;
    // subsampling
    if (c.sub_channels) {
        const std::string s = "encoder.pre_encode.";
        // 3x3 taps go to the device tap-major ([9][C]) so each thread's channel group is contiguous.
        auto taps = [&](const float* src, float** dst) -> ud_status {
            std::vector<float> tr(static_cast<size_t>(9) * C);
            for (int ch = 0; ch < C; ++ch)
                for (int k = 0; k < 9; ++k) tr[static_cast<size_t>(k) * C + ch] = src[ch * 9 + k];
            return upload_f32(e, tr.data(), tr.size(), dst);
        };
        UD_TRY(need(t, s + "conv.0.weight", {C, 1, 3, 3}, &p)); UD_TRY(taps(p, &e->c0_w));
        UD_TRY(need(t, s + "conv.0.bias", {C}, &p)); UD_TRY(upload_f32(e, p, C, &e->c0_b));
        UD_TRY(need(t, s + "conv.2.weight", {C, 1, 3, 3}, &p)); UD_TRY(taps(p, &e->c2_w));
        UD_TRY(need(t, s + "conv.2.bias", {C}, &p)); UD_TRY(upload_f32(e, p, C, &e->c2_b));
        UD_TRY(need(t, s + "conv.3.weight", {C, C, 1, 1}, &p)); UD_TRY(upload_gemm(e, stg, {p}, {C}, C, e->c3));
        UD_TRY(need(t, s + "conv.3.bias", {C}, &p)); UD_TRY(upload_f32(e, p, C, &e->c3_b));
        UD_TRY(need(t, s + "conv.5.weight", {C, 1, 3, 3}, &p)); UD_TRY(taps(p, &e->c5_w));
        UD_TRY(need(t, s + "conv.5.bias", {C}, &p)); UD_TRY(upload_f32(e, p, C, &e->c5_b));
        UD_TRY(need(t, s + "conv.6.weight", {C, C, 1, 1}, &p)); UD_TRY(upload_gemm(e, stg, {p}, {C}, C, e->c6));
        UD_TRY(need(t, s + "conv.6.bias", {C}, &p)); UD_TRY(upload_f32(e, p, C, &e->c6_b));
        // pre_encode.out: checkpoint columns are c*F3 + f (channel-major flatten); the engine's activations are
        // channel-last, so permute to f*C + c (FastConformer.swift:78-94 does the same).
        const int F3 = e->F3;
        UD_TRY(need(t, s + "out.weight", {D, C * F3}, &p));
        std::vector<float> perm(static_cast<size_t>(D) * C * F3);
        for (int o = 0; o < D; ++o)
            for (int ch = 0; ch < C; ++ch)
                for (int f = 0; f < F3; ++f)
                    perm[static_cast<size_t>(o) * C * F3 + f * C + ch] = p[static_cast<size_t>(o) * C * F3 + ch * F3 + f];
        UD_TRY(upload_gemm(e, stg, {perm.data()}, {D}, C * F3, e->sub_out));
        UD_TRY(need(t, s + "out.bias", {D}, &p)); UD_TRY(upload_f32(e, p, D, &e->out_b));
    }
    // layers
    const int tmax = e->tmax;
    const int n_rel = L + 2 * tmax - 1;
    std::vector<float> pe = sinusoid_rows(-(tmax - 1), L + tmax - 1, D);
    float *pe_d = nullptr, *ptab_f = nullptr;
    UD_TRY(dalloc(e, &pe_d, pe.size()));
    UD_TRY(dalloc(e, &ptab_f, pe.size()));
    UD_CK(cudaMemcpyAsync(pe_d, pe.data(), pe.size() * sizeof(float), cudaMemcpyHostToDevice, e->stream));
    e->layers.assign(c.n_layers, LayerW{});
    for (int l = 0; l < c.n_layers; ++l) {
        LayerW& w = e->layers[l];
        const std::string s = "encoder.layers." + std::to_string(l) + ".";
        auto vec = [&](const std::string& nm, int len, float** dst) -> ud_status {
            const float* q;
            UD_TRY(need(t, s + nm, {len}, &q));
            return upload_f32(e, q, len, dst);
        };
        UD_TRY(vec("norm_feed_forward1.weight", D, &w.ln_ff1_g)); UD_TRY(vec("norm_feed_forward1.bias", D, &w.ln_ff1_b));
        UD_TRY(vec("norm_self_att.weight", D, &w.ln_att_g)); UD_TRY(vec("norm_self_att.bias", D, &w.ln_att_b));
        UD_TRY(vec("norm_conv.weight", D, &w.ln_conv_g)); UD_TRY(vec("norm_conv.bias", D, &w.ln_conv_b));
        UD_TRY(vec("conv.batch_norm.weight", D, &w.ln_cbn_g)); UD_TRY(vec("conv.batch_norm.bias", D, &w.ln_cbn_b));
        UD_TRY(vec("norm_feed_forward2.weight", D, &w.ln_ff2_g)); UD_TRY(vec("norm_feed_forward2.bias", D, &w.ln_ff2_b));
        UD_TRY(vec("norm_out.weight", D, &w.ln_out_g)); UD_TRY(vec("norm_out.bias", D, &w.ln_out_b));
        const float *a, *b2, *c3;
        UD_TRY(need(t, s + "feed_forward1.linear1.weight", {F, D}, &a)); UD_TRY(upload_gemm(e, stg, {a}, {F}, D, w.ff1_w1));
        UD_TRY(need(t, s + "feed_forward1.linear2.weight", {D, F}, &a)); UD_TRY(upload_gemm(e, stg, {a}, {D}, F, w.ff1_w2));
        UD_TRY(need(t, s + "feed_forward2.linear1.weight", {F, D}, &a)); UD_TRY(upload_gemm(e, stg, {a}, {F}, D, w.ff2_w1));
        UD_TRY(need(t, s + "feed_forward2.linear2.weight", {D, F}, &a)); UD_TRY(upload_gemm(e, stg, {a}, {D}, F, w.ff2_w2));
        UD_TRY(need(t, s + "self_attn.linear_q.weight", {D, D}, &a));
        UD_TRY(need(t, s + "self_attn.linear_k.weight", {D, D}, &b2));
        UD_TRY(need(t, s + "self_attn.linear_v.weight", {D, D}, &c3));
        UD_TRY(upload_gemm(e, stg, {a, b2, c3}, {D, D, D}, D, w.wqkv));
        UD_TRY(need(t, s + "self_attn.linear_out.weight", {D, D}, &a)); UD_TRY(upload_gemm(e, stg, {a}, {D}, D, w.wo));
        UD_TRY(need(t, s + "conv.pointwise_conv1.weight", {2 * D, D, 1}, &a)); UD_TRY(upload_gemm(e, stg, {a}, {2 * D}, D, w.pw1));
        UD_TRY(need(t, s + "conv.pointwise_conv2.weight", {D, D, 1}, &a)); UD_TRY(upload_gemm(e, stg, {a}, {D}, D, w.pw2));
        UD_TRY(need(t, s + "conv.depthwise_conv.weight", {D, 1, e->KC}, &a));
        {   // tap-major [KC][D] so a thread's channel pair reads each tap with one 8-byte load
            std::vector<float> tm(static_cast<size_t>(D) * e->KC);
            for (int c = 0; c < D; ++c)
                for (int k = 0; k < e->KC; ++k) tm[static_cast<size_t>(k) * D + c] = a[static_cast<size_t>(c) * e->KC + k];
            UD_TRY(upload_f32(e, tm.data(), tm.size(), &w.dw));
            UD_CK(cudaStreamSynchronize(e->stream));   // tm is a temporary
        }
        UD_TRY(need(t, s + "self_attn.pos_bias_u", {H, DK}, &a)); UD_TRY(upload_f32(e, a, D, &w.pos_u));
        UD_TRY(need(t, s + "self_attn.pos_bias_v", {H, DK}, &a)); UD_TRY(upload_f32(e, a, D, &w.pos_v));
        // Projected position table P = sinusoid(rel) . W_pos^T in fp32, stored in the engine dtype.
        UD_TRY(need(t, s + "self_attn.linear_pos.weight", {D, D}, &a));
        UD_CK(cudaMemcpyAsync(stg.p, a, sizeof(float) * D * D, cudaMemcpyHostToDevice, e->stream));
        GemmEpilogue gp;
        gp.out = ptab_f;
        gp.ldo = D;
        gemm_simt<float, float>(pe_d, D, stg.p, n_rel, D, D, gp, e->stream);
        UD_TRY(dalloc_bytes(e, &w.ptab, static_cast<size_t>(n_rel) * D * e->esz));
        if (e->bf) {
            f32_to_bf16(ptab_f, static_cast<bf16*>(w.ptab), static_cast<size_t>(n_rel) * D, e->stream);
            w.has_pmap = make_tma_bf16(w.pmap, w.ptab, n_rel, D, D, 128);
        }
        else UD_CK(cudaMemcpyAsync(w.ptab, ptab_f, sizeof(float) * n_rel * D, cudaMemcpyDeviceToDevice, e->stream));
        UD_CK(cudaStreamSynchronize(e->stream));
    }
    // joint + RNN-T
    if (c.joint_dim) {
        const int J = c.joint_dim, V = c.vocab, Hp = c.pred_hidden;
        UD_TRY(need(t, "joint.enc.weight", {J, D}, &p)); UD_TRY(upload_gemm(e, stg, {p}, {J}, D, e->jenc));
        UD_TRY(need(t, "joint.enc.bias", {J}, &p)); UD_TRY(upload_f32(e, p, J, &e->jenc_b));
        RnntWeights& r = e->rw;
        float* q;
        UD_TRY(need(t, "decoder.prediction.embed.weight", {V, Hp}, &p)); UD_TRY(upload_f32(e, p, static_cast<size_t>(V) * Hp, &q)); r.embed = q;
        for (int l = 0; l < c.pred_layers; ++l) {
            const std::string s = "decoder.prediction.dec_rnn.lstm.";
            const std::string sl = std::to_string(l);
            UD_TRY(need(t, s + "weight_ih_l" + sl, {4 * Hp, Hp}, &p)); UD_TRY(upload_f32(e, p, static_cast<size_t>(4) * Hp * Hp, &q)); r.w_ih[l] = q;
            UD_TRY(need(t, s + "weight_hh_l" + sl, {4 * Hp, Hp}, &p)); UD_TRY(upload_f32(e, p, static_cast<size_t>(4) * Hp * Hp, &q)); r.w_hh[l] = q;
            const float *bi, *bh;
            UD_TRY(need(t, s + "bias_ih_l" + sl, {4 * Hp}, &bi));
            UD_TRY(need(t, s + "bias_hh_l" + sl, {4 * Hp}, &bh));
            std::vector<float> bsum(4 * Hp);
            for (int i = 0; i < 4 * Hp; ++i) bsum[i] = bi[i] + bh[i];
            UD_TRY(upload_f32(e, bsum.data(), bsum.size(), &q)); r.bias[l] = q;
        }
        UD_TRY(need(t, "joint.pred.weight", {J, Hp}, &p)); UD_TRY(upload_f32(e, p, static_cast<size_t>(J) * Hp, &q)); r.pred_w = q;
        UD_TRY(need(t, "joint.pred.bias", {J}, &p)); UD_TRY(upload_f32(e, p, J, &q)); r.pred_b = q;
        UD_TRY(need(t, "joint.joint_net.2.weight", {V, J}, &p)); UD_TRY(upload_f32(e, p, static_cast<size_t>(V) * J, &q)); r.out_w = q;
        UD_TRY(need(t, "joint.joint_net.2.bias", {V}, &p)); UD_TRY(upload_f32(e, p, V, &q)); r.out_b = q;
        r.layers = c.pred_layers;
        r.Hp = Hp;
        r.J = J;
        r.V = V;
        r.max_symbols = c.max_symbols;
        // The tensor-core decoder's fp16 pairs of the same weights (kept off if a value is beyond the fp16 range).
        RnntTc& tc = e->rtc;
        tc.weights_ok = false;
        if (e->rscr.tc) {
            bool ok = true;
            UD_TRY(need(t, "decoder.prediction.embed.weight", {V, Hp}, &p));
            for (size_t i = 0; ok && i < static_cast<size_t>(V) * Hp; ++i) ok = std::fabs(p[i]) < 65504.f;
            const size_t nl = static_cast<size_t>(4) * Hp * 2 * Hp;
            std::vector<uint16_t> hi, lo;
            auto up = [&](uint16_t** dst, const std::vector<uint16_t>& v) -> ud_status {
                UD_TRY(dalloc(e, dst, v.size()));
                UD_CK(cudaMemcpyAsync(*dst, v.data(), v.size() * 2, cudaMemcpyHostToDevice, e->stream));
                UD_CK(cudaStreamSynchronize(e->stream));   // v is reused
                return UD_OK;
            };
            for (int l = 0; ok && l < c.pred_layers; ++l) {
                const std::string s = "decoder.prediction.dec_rnn.lstm.";
                const std::string sl = std::to_string(l);
                const float *wi, *wh;
                UD_TRY(need(t, s + "weight_ih_l" + sl, {4 * Hp, Hp}, &wi));
                UD_TRY(need(t, s + "weight_hh_l" + sl, {4 * Hp, Hp}, &wh));
                hi.assign(nl, 0);
                lo.assign(nl, 0);
                ok = rnnt_tc_split_lstm(wi, wh, Hp, hi.data(), lo.data());
                if (ok) { UD_TRY(up(&tc.wl_hi[l], hi)); UD_TRY(up(&tc.wl_lo[l], lo)); }
            }
            const char* names[2] = {"joint.pred.weight", "joint.joint_net.2.weight"};
            const size_t rows[2] = {static_cast<size_t>(J), static_cast<size_t>(V)};
            const size_t cols[2] = {static_cast<size_t>(Hp), static_cast<size_t>(J)};
            uint16_t** his[2] = {&tc.wp_hi, &tc.wo_hi};
            uint16_t** los[2] = {&tc.wp_lo, &tc.wo_lo};
            for (int m = 0; ok && m < 2; ++m) {
                UD_TRY(need(t, names[m], {static_cast<int>(rows[m]), static_cast<int>(cols[m])}, &p));
                hi.assign(rows[m] * cols[m], 0);
                lo.assign(rows[m] * cols[m], 0);
                ok = rnnt_tc_split(p, hi.size(), hi.data(), lo.data());
                if (ok) { UD_TRY(up(his[m], hi)); UD_TRY(up(los[m], lo)); }
            }
            tc.weights_ok = ok;
            tc.bn_lstm = tc.bn_pred = tc.bn_joint = 0;   // weight maps are rebuilt at the next launch
        }
    }
    UD_CK(cudaStreamSynchronize(e->stream));
    UD_CK(cudaGetLastError());
    e->loaded = true;
    return UD_OK;
}

ud_status reset_slot_device(ud_engine* e, int slot) {
    e->slots_h[0] = slot;
    UD_CK(cudaMemcpyAsync(e->slots_d, e->slots_h, sizeof(int), cudaMemcpyHostToDevice, e->stream));
    {
        Launch L_(e, UD_KIND_CACHE);
        if (e->bf) conv_slot_zero<bf16>(e->slots_d, 1, e->cg, e->stream);
        else conv_slot_zero<float>(e->slots_d, 1, e->cg, e->stream);
    }
    if (e->cfg.joint_dim && e->rs.h) {
        Launch L_(e, UD_KIND_RNNT);
        rnnt_reset(e->rs, e->slots_d, 1, e->rw, e->stream);
    }
    UD_CK(cudaStreamSynchronize(e->stream));
    return UD_OK;
}

// ---------------------------------------------------------------- safetensors
struct StEntry {
    std::string name, dtype;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;
};

bool parse_safetensors_header(const std::string& js, std::vector<StEntry>& out) {
    size_t i = 0;
    auto ws = [&] { while (i < js.size() && (js[i] == ' ' || js[i] == '\n' || js[i] == '\r' || js[i] == '\t')) ++i; };
    auto str = [&](std::string& s) -> bool {
        ws();
        if (i >= js.size() || js[i] != '"') return false;
        ++i;
        s.clear();
        while (i < js.size() && js[i] != '"') {
            if (js[i] == '\\' && i + 1 < js.size()) ++i;
            s += js[i++];
        }
        if (i >= js.size()) return false;
        ++i;
        return true;
    };
    auto num = [&](int64_t& v) -> bool {   // a non-negative integer below 2^62 (shapes and byte offsets)
        ws();
        const size_t st = i;
        v = 0;
        while (i < js.size() && isdigit(static_cast<unsigned char>(js[i]))) {
            if (v > (int64_t(1) << 58)) return false;
            v = v * 10 + (js[i++] - '0');
        }
        return i > st;
    };
    auto skip_value = [&]() -> bool {
        ws();
        int depth = 0;
        bool in_str = false;
        for (; i < js.size(); ++i) {
            const char ch = js[i];
            if (in_str) {
                if (ch == '\\') ++i;
                else if (ch == '"') in_str = false;
                continue;
            }
            if (ch == '"') in_str = true;
            else if (ch == '{' || ch == '[') ++depth;
            else if (ch == '}' || ch == ']') {
                if (depth == 0) return true;
                if (--depth == 0) { ++i; return true; }
            } else if (ch == ',' && depth == 0) return true;
        }
        return false;
    };
    ws();
    if (i >= js.size() || js[i] != '{') return false;
    ++i;
    while (true) {
        ws();
        if (i < js.size() && js[i] == '}') return true;
        StEntry e;
        if (!str(e.name)) return false;
        ws();
        if (i >= js.size() || js[i] != ':') return false;
        ++i;
        ws();
        if (e.name == "__metadata__") {
            if (!skip_value()) return false;
        } else {
            if (i >= js.size() || js[i] != '{') return false;
            ++i;
            while (true) {
                ws();
                if (js[i] == '}') { ++i; break; }
                std::string key;
                if (!str(key)) return false;
                ws();
                if (js[i] != ':') return false;
                ++i;
                if (key == "dtype") {
                    if (!str(e.dtype)) return false;
                } else if (key == "shape" || key == "data_offsets") {
                    ws();
                    if (js[i] != '[') return false;
                    ++i;
                    std::vector<int64_t> v;
                    while (true) {
                        ws();
                        if (js[i] == ']') { ++i; break; }
                        int64_t x;
                        if (!num(x)) return false;
                        v.push_back(x);
                        ws();
                        if (js[i] == ',') ++i;
                    }
                    if (key == "shape") e.shape = v;
                    else if (v.size() == 2) { e.begin = v[0]; e.end = v[1]; }
                } else if (!skip_value()) return false;
                ws();
                if (js[i] == ',') ++i;
            }
            out.push_back(e);
        }
        ws();
        if (i < js.size() && js[i] == ',') ++i;
    }
}

float half_to_float(uint16_t h) {
    const uint32_t sign = (h >> 15) & 1, exp = (h >> 10) & 0x1f, man = h & 0x3ff;
    float v;
    if (exp == 0) v = std::ldexp(static_cast<float>(man), -24);
    else if (exp == 31) v = man ? NAN : INFINITY;
    else v = std::ldexp(static_cast<float>(man | 0x400), static_cast<int>(exp) - 25);
    return sign ? -v : v;
}

}  // namespace

// ================================================================= C ABI
// ---- Allocation-free RNN-T decode -------------------------------------------------------------------------
// ud_rnnt_decode_static stages its per-call scratch (the batch entry, the token count, the token buffer and the
// frames) in this fixed block of the module's static device memory instead of the engine workspace. One block
// per device, shared by every engine and thread on that device.
namespace {

constexpr size_t kStaticScratchBytes = 256 * 1024;
constexpr size_t kScrMeta = 0, kScrCount = 128, kScrTokens = 256;   // byte offsets; frames follow the tokens
constexpr int kMaxScratchDevices = 64;

}  // namespace

static __device__ __align__(256) unsigned char g_rnnt_scratch[kStaticScratchBytes];

namespace {

std::mutex g_scratch_mu;
unsigned char* g_scratch_addr[kMaxScratchDevices];   // resolved once per device
int g_live_engines[kMaxScratchDevices];              // engines alive per device

// The resolved address belongs to the device's current context. When the last engine on a device shuts down it is
// forgotten, so that a context the host application re-creates after that (cudaDeviceReset) is resolved afresh.
void scratch_engine_added(int device) {
    if (device < 0 || device >= kMaxScratchDevices) return;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    ++g_live_engines[device];
}
void scratch_engine_removed(int device) {
    if (device < 0 || device >= kMaxScratchDevices) return;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (--g_live_engines[device] <= 0) {
        g_live_engines[device] = 0;
        g_scratch_addr[device] = nullptr;
    }
}

// Rejections record no message: building one could allocate.
ud_status quiet(ud_status s) {
    g_last_error.clear();
    return s;
}

#define UD_CK_QUIET(call)                                  \
    do {                                                   \
        if ((call) != cudaSuccess) return quiet(UD_ERR_CUDA); \
    } while (0)

}  // namespace

namespace ud {
// Lets other host translation units (the streamer) record an error message for ud_last_error.
ud_status host_fail(ud_status s, const char* msg) { return fail(s, msg); }
}  // namespace ud

// Engine properties for the other translation units of the library (C++ linkage, outside the C ABI).
namespace ud {
cudaStream_t engine_stream(ud_engine* e) { return e->stream; }
int engine_device(ud_engine* e) { return e->device; }
int engine_num_sms(ud_engine* e) { return e->num_sms; }
}  // namespace ud

extern "C" {

void ud_config_default(ud_config* c) {
    if (!c) return;
    c->n_layers = 24;
    c->d_model = 1024;
    c->n_heads = 8;
    c->ff_dim = 4096;
    c->conv_kernel = 9;
    c->left_context = 70;
    c->sub_channels = 256;
    c->mel_bins = 128;
    c->joint_dim = 640;
    c->vocab = 1025;
    c->pred_layers = 1;
    c->pred_hidden = 640;
    c->max_symbols = 10;
    c->dtype = UD_DTYPE_BF16;
    c->max_streams = 64;
    c->max_batch = 64;
    c->max_chunk_frames = 16;
    c->page_frames = 16;
    c->n_pages = 0;
}

const char* ud_status_string(ud_status s) {
    switch (s) {
        case UD_OK: return "ok";
        case UD_ERR_INVALID_ARGUMENT: return "invalid argument";
        case UD_ERR_CUDA: return "CUDA error";
        case UD_ERR_OUT_OF_MEMORY: return "out of memory";
        case UD_ERR_NO_STREAM: return "no such stream";
        case UD_ERR_POOL_EXHAUSTED: return "pool exhausted";
        case UD_ERR_WEIGHTS: return "weights error";
        case UD_ERR_NOT_READY: return "not ready";
        case UD_ERR_DEVICE_TIMEOUT: return "device wait expired";
        case UD_ERR_IO: return "I/O error";
        case UD_ERR_UNSUPPORTED: return "unsupported";
    }
    return "unknown";
}

size_t ud_last_error(char* buf, size_t len) {
    if (buf && len) {
        const size_t n = std::min(len - 1, g_last_error.size());
        std::memcpy(buf, g_last_error.data(), n);
        buf[n] = 0;
    }
    return g_last_error.size();
}

ud_status ud_init(const ud_config* cfg, int device, ud_engine** out) {
    g_last_error.clear();
    if (!cfg || !out) return fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    const ud_config& c = *cfg;
    if (c.n_heads <= 0 || c.d_model != c.n_heads * 128 ||
        (c.n_heads != 1 && c.n_heads != 2 && c.n_heads != 4 && c.n_heads != 6 && c.n_heads != 8))
        return fail(UD_ERR_UNSUPPORTED, "this build needs 128-wide heads and d_model in {128,256,512,768,1024}");
    if (c.conv_kernel != 9) return fail(UD_ERR_UNSUPPORTED, "this build supports conv_kernel 9");
    if (c.n_layers < 0 || c.ff_dim <= 0 || c.ff_dim % 128 != 0) return fail(UD_ERR_INVALID_ARGUMENT, "bad layer sizes");
    if (c.left_context < 1 || c.max_chunk_frames < 1 || c.max_chunk_frames > 32)
        return fail(UD_ERR_INVALID_ARGUMENT, "left_context / max_chunk_frames out of range");
    if (c.page_frames < 1 || c.left_context + c.max_chunk_frames + c.page_frames - 1 > kPageSlots * c.page_frames)
        return fail(UD_ERR_INVALID_ARGUMENT, "page ring too small for left_context + max_chunk_frames");
    if (c.dtype != UD_DTYPE_F32 && c.dtype != UD_DTYPE_BF16) return fail(UD_ERR_INVALID_ARGUMENT, "bad dtype");
    if (c.max_streams < 1 || c.max_batch < 1 || c.max_batch > c.max_streams)
        return fail(UD_ERR_INVALID_ARGUMENT, "max_streams / max_batch out of range");
    if (c.sub_channels && (c.sub_channels % 128 != 0 || c.mel_bins < 1))
        return fail(UD_ERR_UNSUPPORTED, "sub_channels must be a multiple of 128");
    if (c.joint_dim && (c.joint_dim % 128 != 0 || c.pred_hidden % 4 != 0 || c.pred_layers < 1 || c.pred_layers > 4 ||
                        c.vocab < 2 || c.max_symbols < 1))
        return fail(UD_ERR_UNSUPPORTED, "RNN-T head sizes not supported");

    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return fail(UD_ERR_CUDA, "cudaSetDevice failed (no CUDA device?)");
    }
    cudaDeviceProp prop;
    UD_CK(cudaGetDeviceProperties(&prop, device));
    if (c.dtype == UD_DTYPE_BF16 && prop.major != 10)
        return fail(UD_ERR_UNSUPPORTED, "the bf16 engine needs an sm_100 (B200) device");

    ud_engine* e = new ud_engine();
    e->cfg = c;
    e->device = device;
    e->num_sms = prop.multiProcessorCount;
    e->bf = c.dtype == UD_DTYPE_BF16;
    e->esz = e->bf ? 2 : 4;
    e->tmax = c.max_chunk_frames;
    e->L = c.left_context;
    e->D = c.d_model;
    e->H = c.n_heads;
    e->F = c.ff_dim;
    e->KC = c.conv_kernel;
    e->C = c.sub_channels;
    e->J = c.joint_dim;
    e->F1 = nxt(c.mel_bins);
    e->F2 = nxt(e->F1);
    e->F3 = nxt(e->F2);
    auto cleanup = [&](ud_status s) {
        std::string keep = g_last_error;
        ud_shutdown(e);
        g_last_error = keep;
        return s;
    };
    if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&e->stream2, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&e->ev_join, cudaEventDisableTiming) != cudaSuccess)
        return cleanup(fail(UD_ERR_CUDA, "cudaStreamCreate failed"));
    if (const char* g = std::getenv("UD_SPLIT")) e->split_min_rows = std::atoi(g);

    const bool sub = c.sub_channels > 0;
    if (sub) {
        int r = 1;
        while (sub_len(r + 1) <= e->tmax + 2) ++r;
        e->max_rows_in = r;
    } else {
        e->max_rows_in = e->tmax;
    }
    e->in_width = sub ? c.mel_bins : e->D;
    e->out_width = c.joint_dim ? c.joint_dim : e->D;
    e->Mcap = c.max_batch * e->tmax;
    const size_t Mc = e->Mcap, D = e->D, es = e->esz, B = c.max_batch;

    // caches
    const int PF = c.page_frames;
    const int per_stream = (e->L + e->tmax + PF - 1 + PF - 1) / PF;
    const int n_pages = c.n_pages > 0 ? c.n_pages : c.max_streams * per_stream;
    ud_status s;
    CacheGeom& cg = e->cg;
    cg.n_layers = c.n_layers;
    cg.n_pages = n_pages;
    cg.page_frames = PF;
    cg.D = e->D;
    cg.L = e->L;
    cg.conv_ring = c.conv_kernel - 1;
    cg.max_streams = c.max_streams;
    const size_t pool_bytes = static_cast<size_t>(std::max(c.n_layers, 1)) * n_pages * PF * D * es;
    if ((s = dalloc_bytes(e, &cg.kpool, pool_bytes)) != UD_OK) return cleanup(s);
    if ((s = dalloc_bytes(e, &cg.vpool, pool_bytes)) != UD_OK) return cleanup(s);
    const size_t conv_bytes = static_cast<size_t>(std::max(c.n_layers, 1)) * c.max_streams * cg.conv_ring * D * es;
    if ((s = dalloc_bytes(e, &cg.conv, conv_bytes)) != UD_OK) return cleanup(s);
    if (cudaMemset(cg.conv, 0, conv_bytes) != cudaSuccess) return cleanup(fail(UD_ERR_CUDA, "cudaMemset failed"));
    e->free_pages.reserve(n_pages);
    for (int p = n_pages - 1; p >= 0; --p) e->free_pages.push_back(p);
    e->slots.assign(c.max_streams, Slot{});
    for (int i = c.max_streams - 1; i >= 0; --i) e->free_slots.push_back(i);

    // workspace
    if ((s = dalloc(e, &e->x, Mc * D)) != UD_OK) return cleanup(s);
    if ((s = dalloc_bytes(e, &e->h, Mc * D * es)) != UD_OK) return cleanup(s);
    if ((s = dalloc_bytes(e, &e->hid, Mc * e->F * es)) != UD_OK) return cleanup(s);
    if ((s = dalloc_bytes(e, &e->qkv, Mc * 3 * D * es)) != UD_OK) return cleanup(s);
    if ((s = dalloc_bytes(e, &e->att, Mc * D * es)) != UD_OK) return cleanup(s);
    if ((s = dalloc_bytes(e, &e->pw, Mc * 2 * D * es)) != UD_OK) return cleanup(s);
    if ((s = dalloc_bytes(e, &e->y, Mc * D * es)) != UD_OK) return cleanup(s);
    if (c.joint_dim && (s = dalloc(e, &e->proj, Mc * c.joint_dim)) != UD_OK) return cleanup(s);
    if (sub) {
        const size_t T2 = nxt(nxt(e->max_rows_in)), T3 = nxt(T2), C = e->C;   // conv0's output is never stored
        if ((s = dalloc_bytes(e, &e->a2, B * T2 * e->F2 * C * es)) != UD_OK) return cleanup(s);
        if ((s = dalloc_bytes(e, &e->a3, B * T2 * e->F2 * C * es)) != UD_OK) return cleanup(s);
        if ((s = dalloc_bytes(e, &e->a4, B * T3 * e->F3 * C * es)) != UD_OK) return cleanup(s);
        if ((s = dalloc_bytes(e, &e->a5, B * T3 * e->F3 * C * es)) != UD_OK) return cleanup(s);
        if ((s = dalloc(e, &e->subout, B * T3 * D)) != UD_OK) return cleanup(s);
    }
    const size_t in_elems = B * e->max_rows_in * e->in_width;
    const size_t out_elems = B * e->tmax * e->out_width;
    const size_t tok_elems = B * e->tmax * c.max_symbols;
    if ((s = dalloc(e, &e->in_stage, in_elems)) != UD_OK) return cleanup(s);
    if ((s = dalloc(e, &e->out_stage, out_elems)) != UD_OK) return cleanup(s);
    if ((s = dalloc(e, &e->tok_dev, tok_elems)) != UD_OK) return cleanup(s);
    if ((s = dalloc(e, &e->ntok_dev, B)) != UD_OK) return cleanup(s);
    if ((s = halloc(e, &e->h_in, in_elems)) != UD_OK) return cleanup(s);
    if ((s = halloc(e, &e->h_ntok, B)) != UD_OK) return cleanup(s);
    const size_t meta_n = std::max<size_t>(B, c.max_streams);
    for (int r = 0; r < ud_engine::kRing; ++r) {
        if ((s = halloc(e, &e->meta_h[r], meta_n)) != UD_OK) return cleanup(s);
        if ((s = dalloc(e, &e->meta_d[r], meta_n)) != UD_OK) return cleanup(s);
        if (cudaEventCreateWithFlags(&e->meta_ev[r], cudaEventDisableTiming) != cudaSuccess)
            return cleanup(fail(UD_ERR_CUDA, "cudaEventCreate failed"));
    }
    if ((s = dalloc(e, &e->meta_graph_d, meta_n)) != UD_OK) return cleanup(s);
    if (const char* g = std::getenv("UD_GRAPHS")) e->graphs_on = std::atoi(g) != 0;
    if (const char* g = std::getenv("UD_TC2")) e->tc2_on = std::atoi(g) != 0;
    if (const char* g = std::getenv("UD_ATTN_TMA")) e->attn_tma_on = std::atoi(g) != 0;
    if (e->bf && c.n_layers > 0 && PF == 16)
        e->attn_maps = make_tma_bf16(e->attn_qkv_map, e->qkv, static_cast<int>(Mc), 3 * e->D, 3 * e->D, 16) &&
                       make_tma_pages(e->attn_k_map, cg.kpool, c.n_layers * n_pages, PF, e->D) &&
                       make_tma_pages(e->attn_v_map, cg.vpool, c.n_layers * n_pages, PF, e->D);
    if ((s = halloc(e, &e->slots_h, meta_n)) != UD_OK) return cleanup(s);
    if ((s = dalloc(e, &e->slots_d, meta_n)) != UD_OK) return cleanup(s);
    if ((s = dalloc(e, &e->err_d, 1)) != UD_OK) return cleanup(s);
    if ((s = halloc(e, &e->err_h, 1)) != UD_OK) return cleanup(s);
    if (cudaMemset(e->err_d, 0, sizeof(int)) != cudaSuccess) return cleanup(fail(UD_ERR_CUDA, "cudaMemset failed"));
    if (c.joint_dim) {
        const size_t S = c.max_streams, Hp = c.pred_hidden, NLp = c.pred_layers;
        RnntState& r = e->rs;
        if ((s = dalloc(e, &r.h, S * NLp * Hp)) != UD_OK) return cleanup(s);
        if ((s = dalloc(e, &r.c, S * NLp * Hp)) != UD_OK) return cleanup(s);
        if ((s = dalloc(e, &r.pend_h, S * NLp * Hp)) != UD_OK) return cleanup(s);
        if ((s = dalloc(e, &r.pend_c, S * NLp * Hp)) != UD_OK) return cleanup(s);
        if ((s = dalloc(e, &r.pend_g, S * c.joint_dim)) != UD_OK) return cleanup(s);
        if ((s = dalloc(e, &r.last_tok, S)) != UD_OK) return cleanup(s);
        if ((s = dalloc(e, &r.pend_valid, S)) != UD_OK) return cleanup(s);
        if (const char* g = std::getenv("UD_RNNT_LOCKSTEP")) e->rnnt_lockstep = std::atoi(g) != 0;
        RnntScratch& q = e->rscr;
        q.max_n = c.max_batch;
        q.max_grid = e->num_sms;
        if (const char* g = std::getenv("UD_RNNT_LOCKSTEP_MAX")) q.lockstep_max_n = std::atoi(g);
        const size_t parts = static_cast<size_t>(q.max_n) * q.max_grid;
        if ((s = dalloc(e, &q.barrier, 1)) != UD_OK) return cleanup(s);
        if ((s = dalloc(e, &q.done_frame, q.max_n)) != UD_OK) return cleanup(s);
        if ((s = dalloc(e, &q.emitted, q.max_n)) != UD_OK) return cleanup(s);
        if ((s = dalloc(e, &q.part_val, parts)) != UD_OK) return cleanup(s);
        if ((s = dalloc(e, &q.part_idx, parts)) != UD_OK) return cleanup(s);
        // Tensor-core decoder rows (UD_RNNT_TC=0 leaves it off; UD_RNNT_TC=n takes batches of n streams and up,
        // 20 by default).
        if (const char* g = std::getenv("UD_RNNT_TC")) q.tc_min_n = std::atoi(g);
        if (q.tc_min_n > 0 && Hp % 64 == 0 && c.joint_dim % 64 == 0 && NLp <= 4) {
            RnntTc& tc = e->rtc;
            tc.n_pad = (q.max_n + 127) / 128 * 128;
            const size_t NP = tc.n_pad;
            for (size_t l = 0; l < NLp; ++l) {
                if ((s = dalloc(e, &tc.xl_hi[l], NP * 2 * Hp)) != UD_OK) return cleanup(s);
                if ((s = dalloc(e, &tc.xl_lo[l], NP * 2 * Hp)) != UD_OK) return cleanup(s);
                cudaMemsetAsync(tc.xl_hi[l], 0, NP * 2 * Hp * 2, e->stream);
                cudaMemsetAsync(tc.xl_lo[l], 0, NP * 2 * Hp * 2, e->stream);
            }
            uint16_t** rows[4] = {&tc.xp_hi, &tc.xp_lo, &tc.xj_hi, &tc.xj_lo};
            const size_t widths[4] = {Hp, Hp, static_cast<size_t>(c.joint_dim), static_cast<size_t>(c.joint_dim)};
            for (int i = 0; i < 4; ++i) {
                if ((s = dalloc(e, rows[i], NP * widths[i])) != UD_OK) return cleanup(s);
                cudaMemsetAsync(*rows[i], 0, NP * widths[i] * 2, e->stream);
            }
            if (rnnt_tc_build_row_maps(tc, static_cast<int>(NLp), static_cast<int>(Hp), c.joint_dim)) q.tc = &tc;
        }
    }
    if (cudaDeviceSynchronize() != cudaSuccess) return cleanup(fail(UD_ERR_CUDA, "device synchronize failed"));
    scratch_engine_added(device);
    e->counted = true;
    *out = e;
    return UD_OK;
}

ud_status ud_shutdown(ud_engine* e) {
    if (!e) return UD_OK;
    cudaSetDevice(e->device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    if (e->stream2) cudaStreamSynchronize(e->stream2);
    for (void* p : e->allocs) cudaFree(p);
    for (void* p : e->host_allocs) cudaFreeHost(p);
    if (e->cstream) cudaStreamSynchronize(e->cstream);
    if (e->ostream) cudaStreamSynchronize(e->ostream);
    for (int r = 0; r < ud_engine::kRing; ++r)
        if (e->meta_ev[r]) cudaEventDestroy(e->meta_ev[r]);
    for (int b = 0; b < 2; ++b)
        for (cudaEvent_t ev : {e->ev_in[b], e->ev_done[b], e->ev_out[b]})
            if (ev) cudaEventDestroy(ev);
    if (e->cstream) cudaStreamDestroy(e->cstream);
    if (e->ostream) cudaStreamDestroy(e->ostream);
    for (cudaEvent_t ev : e->prof_events) cudaEventDestroy(ev);
    for (auto& g : e->graphs) cudaGraphExecDestroy(g.second.exec);
    if (e->stream) cudaStreamDestroy(e->stream);
    if (e->stream2) cudaStreamDestroy(e->stream2);
    for (cudaEvent_t ev : {e->ev_fork, e->ev_join})
        if (ev) cudaEventDestroy(ev);
    if (e->counted) scratch_engine_removed(e->device);
    delete e;
    return UD_OK;
}

ud_status ud_load_weights(ud_engine* e, const ud_weight* table, int n) {
    if (!e || !table || n <= 0) return fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (e->loaded) return fail(UD_ERR_INVALID_ARGUMENT, "weights already loaded");
    UD_CK(cudaSetDevice(e->device));
    return load_weights_impl(e, table, n);
}

ud_status ud_load_safetensors(ud_engine* e, const char* path) {
    if (!e || !path) return fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    FILE* f = std::fopen(path, "rb");
    if (!f) return fail(UD_ERR_IO, std::string("cannot open ") + path);
    uint64_t hlen = 0;
    if (std::fread(&hlen, 8, 1, f) != 1 || hlen > (1ull << 30)) {
        std::fclose(f);
        return fail(UD_ERR_IO, "bad safetensors header length");
    }
    std::string js(hlen, '\0');
    if (std::fread(&js[0], 1, hlen, f) != hlen) {
        std::fclose(f);
        return fail(UD_ERR_IO, "short safetensors header");
    }
    std::vector<StEntry> ents;
    if (!parse_safetensors_header(js, ents)) {
        std::fclose(f);
        return fail(UD_ERR_IO, "cannot parse safetensors header");
    }
    // Tensors of other dtypes (integer counters such as a batch norm's num_batches_tracked) are not weights the
    // engine reads: they are skipped, and a needed tensor stored that way is reported missing.
    std::vector<std::vector<float>> data(ents.size());
    std::vector<ud_weight> table;
    table.reserve(ents.size());
    const uint64_t base = 8 + hlen;
    for (size_t k = 0; k < ents.size(); ++k) {
        const StEntry& en = ents[k];
        int64_t count = 1;
        for (int64_t d : en.shape) count *= d;
        const int esz = en.dtype == "F32" ? 4 : (en.dtype == "F16" || en.dtype == "BF16") ? 2 : 0;
        if (!esz) continue;
        if (en.shape.size() > 4 || en.end - en.begin != static_cast<uint64_t>(count) * esz) {
            std::fclose(f);
            return fail(UD_ERR_IO, "bad tensor " + en.name + " (" + en.dtype + ")");
        }
        std::vector<uint8_t> raw(en.end - en.begin);
        if (std::fseek(f, static_cast<long>(base + en.begin), SEEK_SET) != 0 ||
            std::fread(raw.data(), 1, raw.size(), f) != raw.size()) {
            std::fclose(f);
            return fail(UD_ERR_IO, "short read of " + en.name);
        }
        data[k].resize(count);
        for (int64_t i = 0; i < count; ++i) {
            if (esz == 4) {
                std::memcpy(&data[k][i], &raw[i * 4], 4);
            } else {
                uint16_t hv;
                std::memcpy(&hv, &raw[i * 2], 2);
                if (en.dtype == "F16") {
                    data[k][i] = half_to_float(hv);
                } else {
                    const uint32_t bits = static_cast<uint32_t>(hv) << 16;
                    std::memcpy(&data[k][i], &bits, 4);
                }
            }
        }
        ud_weight w{};
        w.name = ents[k].name.c_str();
        w.data = data[k].data();
        w.ndim = static_cast<int>(en.shape.size());
        for (size_t d = 0; d < en.shape.size(); ++d) w.shape[d] = en.shape[d];
        table.push_back(w);
    }
    std::fclose(f);
    if (table.empty()) return fail(UD_ERR_WEIGHTS, "no F32/F16/BF16 tensors in the file");
    return ud_load_weights(e, table.data(), static_cast<int>(table.size()));
}

ud_status ud_stream_open(ud_engine* e, int lookahead, ud_stream_id* out) {
    if (!e || !out) return fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (lookahead < 0) return fail(UD_ERR_INVALID_ARGUMENT, "negative lookahead");
    if (e->free_slots.empty()) return fail(UD_ERR_POOL_EXHAUSTED, "no free stream slot");
    UD_CK(cudaSetDevice(e->device));
    const int id = e->free_slots.back();
    Slot& s = e->slots[id];
    s.reset();
    s.lookahead = lookahead;
    UD_TRY(reset_slot_device(e, id));
    e->free_slots.pop_back();
    s.open = true;
    *out = id;
    return UD_OK;
}

ud_status ud_stream_close(ud_engine* e, ud_stream_id id) {
    if (!e) return fail(UD_ERR_INVALID_ARGUMENT, "NULL engine");
    if (id < 0 || id >= e->cfg.max_streams || !e->slots[id].open) return fail(UD_ERR_NO_STREAM, "unknown stream");
    Slot& s = e->slots[id];
    free_all_pages(e, s);
    s.open = false;
    e->free_slots.push_back(id);
    return UD_OK;
}

ud_status ud_step_batch_device(ud_engine* e, int n, const ud_stream_id* ids, const float* mel_dev, int rows_stride,
                               const int* n_rows, const int* valid_rows, const int* keep_all, float* proj_dev,
                               int* frames_out, int32_t* tokens_dev, int* n_tokens_dev) {
    if (!e) return fail(UD_ERR_INVALID_ARGUMENT, "NULL engine");
    if (tokens_dev && !n_tokens_dev) return fail(UD_ERR_INVALID_ARGUMENT, "n_tokens_dev is NULL");
    if (!mel_dev || !proj_dev || !n_rows) return fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (n < 1 || n > e->cfg.max_batch) return fail(UD_ERR_INVALID_ARGUMENT, "batch size out of range");
    UD_CK(cudaSetDevice(e->device));
    UD_TRY(drain_async(e));
    int rows_max = 1;
    for (int i = 0; i < n; ++i) {
        if (n_rows[i] < 1 || n_rows[i] > e->max_rows_in || n_rows[i] > rows_stride)
            return fail(UD_ERR_INVALID_ARGUMENT, "n_rows out of range");
        rows_max = std::max(rows_max, n_rows[i]);
    }
    // Stage the input into the engine's fixed buffer (the step, or its captured graph, reads it from there).
    const size_t W = e->in_width;
    UD_CK(cudaMemcpy2DAsync(e->in_stage, sizeof(float) * W * e->max_rows_in, mel_dev, sizeof(float) * W * rows_stride,
                            sizeof(float) * W * rows_max, n, cudaMemcpyDeviceToDevice, e->stream));
    UD_TRY(run_batch(e, n, ids, e->in_stage, e->max_rows_in, n_rows, valid_rows, keep_all, e->out_stage, frames_out,
                     tokens_dev ? e->tok_dev : nullptr, e->ntok_dev, true));
    UD_CK(cudaMemcpyAsync(proj_dev, e->out_stage, sizeof(float) * n * e->tmax * e->out_width, cudaMemcpyDeviceToDevice,
                          e->stream));
    if (tokens_dev) {
        UD_CK(cudaMemcpyAsync(tokens_dev, e->tok_dev, sizeof(int32_t) * n * e->tmax * e->cfg.max_symbols,
                              cudaMemcpyDeviceToDevice, e->stream));
        UD_CK(cudaMemcpyAsync(n_tokens_dev, e->ntok_dev, sizeof(int) * n, cudaMemcpyDeviceToDevice, e->stream));
    }
    return UD_OK;
}

ud_status ud_step_batch(ud_engine* e, int n, const ud_stream_id* ids, const float* const* mel, const int* n_rows,
                        const int* valid_rows, const int* keep_all, float* proj_out, int* frames_out,
                        int32_t* tokens_out, int* n_tokens_out) {
    if (!e || !mel || !n_rows || (!proj_out && !tokens_out)) return fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (n < 1 || n > e->cfg.max_batch) return fail(UD_ERR_INVALID_ARGUMENT, "batch size out of range");
    if (tokens_out && !n_tokens_out) return fail(UD_ERR_INVALID_ARGUMENT, "n_tokens_out is NULL");
    UD_CK(cudaSetDevice(e->device));
    const int stride = e->max_rows_in;
    int rows_max = 1;
    for (int i = 0; i < n; ++i) {
        if (!mel[i]) return fail(UD_ERR_INVALID_ARGUMENT, "NULL input rows");
        if (n_rows[i] < 1 || n_rows[i] > e->max_rows_in)
            return fail(UD_ERR_INVALID_ARGUMENT, "n_rows out of range");
        rows_max = std::max(rows_max, n_rows[i]);
    }
    const int W = e->in_width;
    UD_TRY(drain_async(e));
    // The pinned staging buffer may still be read by a previous asynchronous call.
    UD_CK(cudaStreamSynchronize(e->stream));
    // Rows of all streams in one caller buffer at a fixed stride: one strided copy straight from it (a DMA when
    // the caller's memory is pinned). Otherwise gather through the pinned staging buffer.
    bool uniform = true;
    const ptrdiff_t sstride = n > 1 ? mel[1] - mel[0] : static_cast<ptrdiff_t>(W) * stride;
    for (int i = 1; i < n && uniform; ++i) uniform = mel[i] - mel[0] == sstride * i;
    uniform = uniform && sstride >= static_cast<ptrdiff_t>(W) * rows_max;
    if (uniform) {
        UD_CK(cudaMemcpy2DAsync(e->in_stage, sizeof(float) * W * stride, mel[0], sizeof(float) * sstride,
                                sizeof(float) * W * rows_max, n, cudaMemcpyHostToDevice, e->stream));
    } else {
        for (int i = 0; i < n; ++i)
            std::memcpy(e->h_in + static_cast<size_t>(i) * stride * W, mel[i], sizeof(float) * n_rows[i] * W);
        UD_CK(cudaMemcpy2DAsync(e->in_stage, sizeof(float) * W * stride, e->h_in, sizeof(float) * W * stride,
                                sizeof(float) * W * rows_max, n, cudaMemcpyHostToDevice, e->stream));
    }
    std::vector<int> frames(n);
    UD_TRY(run_batch(e, n, ids, e->in_stage, stride, n_rows, valid_rows, keep_all, e->out_stage, frames.data(),
                     tokens_out ? e->tok_dev : nullptr, e->ntok_dev, true));
    const size_t out_n = static_cast<size_t>(n) * e->tmax * e->out_width;
    if (proj_out)
        UD_CK(cudaMemcpyAsync(proj_out, e->out_stage, sizeof(float) * out_n, cudaMemcpyDeviceToHost, e->stream));
    if (tokens_out) {
        UD_CK(cudaMemcpyAsync(tokens_out, e->tok_dev, sizeof(int32_t) * n * e->tmax * e->cfg.max_symbols,
                              cudaMemcpyDeviceToHost, e->stream));
        UD_CK(cudaMemcpyAsync(n_tokens_out, e->ntok_dev, sizeof(int) * n, cudaMemcpyDeviceToHost, e->stream));
    }
    UD_TRY(check_device_error(e));
    if (frames_out) std::memcpy(frames_out, frames.data(), sizeof(int) * n);
    return UD_OK;
}

ud_status ud_step_batch_async(ud_engine* e, int n, const ud_stream_id* ids, const float* const* mel, const int* n_rows,
                              const int* valid_rows, const int* keep_all, float* proj_out, int* frames_out,
                              int32_t* tokens_out, int* n_tokens_out) {
    if (!e || !mel || !n_rows || (!proj_out && !tokens_out)) return fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (n < 1 || n > e->cfg.max_batch) return fail(UD_ERR_INVALID_ARGUMENT, "batch size out of range");
    if (tokens_out && !n_tokens_out) return fail(UD_ERR_INVALID_ARGUMENT, "n_tokens_out is NULL");
    UD_CK(cudaSetDevice(e->device));
    const int stride = e->max_rows_in;
    int rows_max = 1;
    for (int i = 0; i < n; ++i) {
        if (!mel[i]) return fail(UD_ERR_INVALID_ARGUMENT, "NULL input rows");
        if (n_rows[i] < 1 || n_rows[i] > e->max_rows_in)
            return fail(UD_ERR_INVALID_ARGUMENT, "n_rows out of range");
        rows_max = std::max(rows_max, n_rows[i]);
    }
    UD_TRY(async_setup(e));
    // Step k uses staging buffer k % 2. Step k - 2, its last user, completed before call k - 1 returned.
    const int b = static_cast<int>(e->async_issued & 1);
    float* in_d = b ? e->in_stage2 : e->in_stage;
    float* out_d = b ? e->out_stage2 : e->out_stage;
    float* h_in = b ? e->h_in2 : e->h_in;
    int32_t* tok_d = b ? e->tok_dev2 : e->tok_dev;
    int* ntok_d = b ? e->ntok_dev2 : e->ntok_dev;
    const int W = e->in_width;
    bool uniform = true;
    const ptrdiff_t sstride = n > 1 ? mel[1] - mel[0] : static_cast<ptrdiff_t>(W) * stride;
    for (int i = 1; i < n && uniform; ++i) uniform = mel[i] - mel[0] == sstride * i;
    uniform = uniform && sstride >= static_cast<ptrdiff_t>(W) * rows_max;
    const float* src = mel[0];
    size_t spitch = sizeof(float) * sstride;
    if (!uniform) {
        for (int i = 0; i < n; ++i)
            std::memcpy(h_in + static_cast<size_t>(i) * stride * W, mel[i], sizeof(float) * n_rows[i] * W);
        src = h_in;
        spitch = sizeof(float) * W * stride;
    }
    UD_CK(cudaMemcpy2DAsync(in_d, sizeof(float) * W * stride, src, spitch, sizeof(float) * W * rows_max, n,
                            cudaMemcpyHostToDevice, e->cstream));
    UD_CK(cudaEventRecord(e->ev_in[b], e->cstream));
    UD_CK(cudaStreamWaitEvent(e->stream, e->ev_in[b], 0));
    std::vector<int> frames(n);
    UD_TRY(run_batch(e, n, ids, in_d, stride, n_rows, valid_rows, keep_all, out_d, frames.data(),
                     tokens_out ? tok_d : nullptr, ntok_d, true));
    UD_CK(cudaMemcpyAsync(e->err_async_h + b, e->err_d, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    UD_CK(cudaEventRecord(e->ev_done[b], e->stream));
    UD_CK(cudaStreamWaitEvent(e->ostream, e->ev_done[b], 0));
    const size_t out_n = static_cast<size_t>(n) * e->tmax * e->out_width;
    if (proj_out)
        UD_CK(cudaMemcpyAsync(proj_out, out_d, sizeof(float) * out_n, cudaMemcpyDeviceToHost, e->ostream));
    if (tokens_out) {
        UD_CK(cudaMemcpyAsync(tokens_out, tok_d, sizeof(int32_t) * n * e->tmax * e->cfg.max_symbols,
                              cudaMemcpyDeviceToHost, e->ostream));
        UD_CK(cudaMemcpyAsync(n_tokens_out, ntok_d, sizeof(int) * n, cudaMemcpyDeviceToHost, e->ostream));
    }
    UD_CK(cudaEventRecord(e->ev_out[b], e->ostream));
    ++e->async_issued;
    if (frames_out) std::memcpy(frames_out, frames.data(), sizeof(int) * n);
    // complete the previous step: its outputs are in place, its buffers free for the next call
    if (e->async_issued - e->async_completed > 1) {
        const int pb = b ^ 1;
        UD_CK(cudaEventSynchronize(e->ev_out[pb]));
        ++e->async_completed;
        if (e->err_async_h[pb] != 0) return device_error_status(e, e->err_async_h[pb]);
    }
    return UD_OK;
}

ud_status ud_step_sync(ud_engine* e) {
    if (!e) return fail(UD_ERR_INVALID_ARGUMENT, "NULL engine");
    UD_CK(cudaSetDevice(e->device));
    return drain_async(e);
}

ud_status ud_stream_step(ud_engine* e, ud_stream_id id, const float* mel, int n_rows, int valid_rows, int keep_all,
                         float* proj_out, int* frames_out) {
    if (!e || !mel || !proj_out) return fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    const float* ptrs[1] = {mel};
    int fr = 0;
    if (!e->loaded) return fail(UD_ERR_NOT_READY, "weights not loaded");
    std::vector<float> tmp(static_cast<size_t>(e->tmax) * e->out_width);
    UD_TRY(ud_step_batch(e, 1, &id, ptrs, &n_rows, &valid_rows, &keep_all, tmp.data(), &fr, nullptr, nullptr));
    std::memcpy(proj_out, tmp.data(), sizeof(float) * fr * e->out_width);
    if (frames_out) *frames_out = fr;
    return UD_OK;
}

ud_status ud_rnnt_decode(ud_engine* e, ud_stream_id id, const float* f, int frames, int32_t* tokens_out,
                         int* n_tokens_out) {
    if (!e || !f || !tokens_out || !n_tokens_out) return fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (!e->loaded) return fail(UD_ERR_NOT_READY, "weights not loaded");
    if (!e->cfg.joint_dim) return fail(UD_ERR_INVALID_ARGUMENT, "no RNN-T head in this configuration");
    UD_TRY(check_ids(e, 1, &id));
    if (frames < 0 || frames > e->Mcap) return fail(UD_ERR_INVALID_ARGUMENT, "frames out of range");
    *n_tokens_out = 0;
    if (frames == 0) return UD_OK;
    UD_CK(cudaSetDevice(e->device));
    UD_CK(cudaStreamSynchronize(e->stream));
    int mi = 0;
    BatchEntry* mh = next_meta_host(e, &mi);
    std::memset(&mh[0], 0, sizeof(BatchEntry));
    mh[0].slot = id;
    mh[0].keep = frames;
    mh[0].T = frames;
    UD_TRY(upload_meta(e, mi, 1));
    UD_CK(cudaMemcpyAsync(e->proj, f, sizeof(float) * frames * e->J, cudaMemcpyHostToDevice, e->stream));
    // The token buffer holds max_batch * tmax * max_symbols ids; one stream may use all of it.
    const int cap = e->cfg.max_batch * e->tmax * e->cfg.max_symbols;
    if (frames * e->cfg.max_symbols > cap) return fail(UD_ERR_INVALID_ARGUMENT, "too many frames for one call");
    {
        Launch L_(e, UD_KIND_RNNT);
        rnnt_greedy(e->rw, e->rs, e->proj, e->J, e->meta_d[mi], 1, e->tok_dev, cap, e->ntok_dev,
                    e->rnnt_lockstep ? &e->rscr : nullptr, e->num_sms, e->err_d, e->stream);
    }
    UD_CK(cudaGetLastError());
    UD_CK(cudaMemcpyAsync(e->h_ntok, e->ntok_dev, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    UD_CK(cudaStreamSynchronize(e->stream));
    UD_TRY(check_device_error(e));
    const int nt = e->h_ntok[0];
    UD_CK(cudaMemcpyAsync(tokens_out, e->tok_dev, sizeof(int32_t) * nt, cudaMemcpyDeviceToHost, e->stream));
    UD_CK(cudaStreamSynchronize(e->stream));
    *n_tokens_out = nt;
    return UD_OK;
}

ud_status ud_rnnt_decode_static(ud_engine* e, ud_stream_id id, const float* f, int frames, int32_t* tokens_out,
                                int* n_tokens_out) {
    if (!e || !f || !tokens_out || !n_tokens_out) return quiet(UD_ERR_INVALID_ARGUMENT);
    if (!e->loaded) return quiet(UD_ERR_NOT_READY);
    if (!e->cfg.joint_dim) return quiet(UD_ERR_INVALID_ARGUMENT);
    if (id < 0 || id >= e->cfg.max_streams || !e->slots[id].open) return quiet(UD_ERR_INVALID_ARGUMENT);
    if (frames < 0 || e->device < 0 || e->device >= kMaxScratchDevices) return quiet(UD_ERR_INVALID_ARGUMENT);
    const size_t tok_cap = static_cast<size_t>(frames) * e->cfg.max_symbols;
    const size_t feat_off = (kScrTokens + sizeof(int32_t) * tok_cap + 255) & ~static_cast<size_t>(255);
    const size_t feat_bytes = sizeof(float) * static_cast<size_t>(frames) * e->J;
    if (feat_off + feat_bytes > kStaticScratchBytes) return quiet(UD_ERR_INVALID_ARGUMENT);   // beyond the block
    *n_tokens_out = 0;
    if (frames == 0) return UD_OK;
    UD_CK_QUIET(cudaSetDevice(e->device));
    unsigned char* scr = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_scratch_mu);
        if (!g_scratch_addr[e->device]) {
            void* p = nullptr;
            UD_CK_QUIET(cudaGetSymbolAddress(&p, g_rnnt_scratch));
            g_scratch_addr[e->device] = static_cast<unsigned char*>(p);
        }
        scr = g_scratch_addr[e->device];
    }
    BatchEntry* meta = reinterpret_cast<BatchEntry*>(scr + kScrMeta);
    int* count = reinterpret_cast<int*>(scr + kScrCount);
    int32_t* tokens = reinterpret_cast<int32_t*>(scr + kScrTokens);
    float* feats = reinterpret_cast<float*>(scr + feat_off);
    BatchEntry me;
    std::memset(&me, 0, sizeof(me));
    me.slot = id;
    me.keep = frames;
    me.T = frames;
    // The count must read zero if the kernel never ran; the kernel overwrites it and fills tokens [0, count).
    UD_CK_QUIET(cudaMemcpyAsync(meta, &me, sizeof(me), cudaMemcpyHostToDevice, e->stream));
    UD_CK_QUIET(cudaMemsetAsync(count, 0, sizeof(int), e->stream));
    UD_CK_QUIET(cudaMemcpyAsync(feats, f, feat_bytes, cudaMemcpyHostToDevice, e->stream));
    rnnt_greedy(e->rw, e->rs, feats, e->J, meta, 1, tokens, static_cast<int>(tok_cap), count,
                e->rnnt_lockstep ? &e->rscr : nullptr, e->num_sms, e->err_d, e->stream);
    e->launches++;
    UD_CK_QUIET(cudaGetLastError());
    int nt = 0;
    UD_CK_QUIET(cudaMemcpyAsync(&nt, count, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    UD_CK_QUIET(cudaMemcpyAsync(e->err_h, e->err_d, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    UD_CK_QUIET(cudaStreamSynchronize(e->stream));
    // A bounded device wait that expired (a decoder's grid barrier) or an input the kernel rejected ends the kernel
    // early: the tokens are incomplete, so the call fails with the status device_error_status gives the same code,
    // and the error word is cleared so that the next call starts clean.
    if (const int code = *e->err_h) {
        UD_CK_QUIET(cudaMemsetAsync(e->err_d, 0, sizeof(int), e->stream));
        UD_CK_QUIET(cudaStreamSynchronize(e->stream));
        return quiet((code == DEV_BAD_PAGE || code == DEV_RANGE_F16) ? UD_ERR_INVALID_ARGUMENT : UD_ERR_DEVICE_TIMEOUT);
    }
    if (nt < 0 || static_cast<size_t>(nt) > tok_cap) return quiet(UD_ERR_CUDA);
    if (nt > 0) {
        UD_CK_QUIET(cudaMemcpyAsync(tokens_out, tokens, sizeof(int32_t) * nt, cudaMemcpyDeviceToHost, e->stream));
        UD_CK_QUIET(cudaStreamSynchronize(e->stream));
    }
    *n_tokens_out = nt;
    return UD_OK;
}

ud_status ud_cache_append(ud_engine* e, int n, const ud_stream_id* ids, int k, const void* kv_rows,
                          const void* conv_rows) {
    if (!e) return fail(UD_ERR_INVALID_ARGUMENT, "NULL engine");
    UD_TRY(check_ids(e, n, ids));
    if (k < 1 || k > e->tmax) return fail(UD_ERR_INVALID_ARGUMENT, "k out of range");
    UD_CK(cudaSetDevice(e->device));
    int mi = 0;
    BatchEntry* mh = next_meta_host(e, &mi);
    std::vector<std::pair<Slot*, int>> undo;
    for (int i = 0; i < n; ++i) {
        Slot& s = e->slots[ids[i]];
        if (kv_rows) {
            ud_status st = map_pages(e, s, k, undo);
            if (st != UD_OK) {
                undo_pages(e, undo);
                return st;
            }
        }
        std::memset(&mh[i], 0, sizeof(BatchEntry));
        mh[i].slot = ids[i];
        mh[i].head = s.head;
        mh[i].cache_len = s.cache_len;
        mh[i].T = k;
        std::memcpy(mh[i].pages, s.pages, sizeof(mh[i].pages));
    }
    UD_TRY(upload_meta(e, mi, n));
    {
    Launch L_(e, UD_KIND_CACHE);
    if (e->bf)
        cache_append<bf16>(static_cast<const bf16*>(kv_rows), static_cast<const bf16*>(conv_rows), k, e->meta_d[mi], n,
                           e->cg, e->err_d, e->stream);
    else
        cache_append<float>(static_cast<const float*>(kv_rows), static_cast<const float*>(conv_rows), k, e->meta_d[mi],
                            n, e->cg, e->err_d, e->stream);
    }
    UD_CK(cudaGetLastError());
    return UD_OK;
}

ud_status ud_cache_roll(ud_engine* e, int n, const ud_stream_id* ids, int k) {
    if (!e) return fail(UD_ERR_INVALID_ARGUMENT, "NULL engine");
    UD_TRY(check_ids(e, n, ids));
    if (k < 1 || k > e->tmax) return fail(UD_ERR_INVALID_ARGUMENT, "k out of range");
    for (int i = 0; i < n; ++i) {
        Slot& s = e->slots[ids[i]];
        s.head += k;
        s.cache_len = std::min(s.cache_len + k, e->L);
        free_out_of_window(e, s);
    }
    return UD_OK;
}

ud_status ud_cache_gather(ud_engine* e, int n, const ud_stream_id* ids, void* kv_out, void* conv_out) {
    if (!e) return fail(UD_ERR_INVALID_ARGUMENT, "NULL engine");
    UD_TRY(check_ids(e, n, ids));
    UD_CK(cudaSetDevice(e->device));
    int mi = 0;
    BatchEntry* mh = next_meta_host(e, &mi);
    for (int i = 0; i < n; ++i) {
        const Slot& s = e->slots[ids[i]];
        std::memset(&mh[i], 0, sizeof(BatchEntry));
        mh[i].slot = ids[i];
        mh[i].head = s.head;
        mh[i].cache_len = s.cache_len;
        std::memcpy(mh[i].pages, s.pages, sizeof(mh[i].pages));
    }
    UD_TRY(upload_meta(e, mi, n));
    {
    Launch L_(e, UD_KIND_CACHE);
    if (e->bf)
        cache_gather<bf16>(static_cast<bf16*>(kv_out), static_cast<bf16*>(conv_out), e->meta_d[mi], n, e->cg, e->err_d,
                           e->stream);
    else
        cache_gather<float>(static_cast<float*>(kv_out), static_cast<float*>(conv_out), e->meta_d[mi], n, e->cg,
                            e->err_d, e->stream);
    }
    UD_CK(cudaGetLastError());
    return UD_OK;
}

ud_status ud_cache_evict(ud_engine* e, int n, const ud_stream_id* ids) {
    if (!e) return fail(UD_ERR_INVALID_ARGUMENT, "NULL engine");
    UD_TRY(check_ids(e, n, ids));
    UD_CK(cudaSetDevice(e->device));
    for (int i = 0; i < n; ++i) {
        Slot& s = e->slots[ids[i]];
        free_all_pages(e, s);
        const int la = s.lookahead;
        s.reset();
        s.lookahead = la;
        e->slots_h[i] = ids[i];
    }
    UD_CK(cudaStreamSynchronize(e->stream));
    UD_CK(cudaMemcpyAsync(e->slots_d, e->slots_h, sizeof(int) * n, cudaMemcpyHostToDevice, e->stream));
    {
        Launch L_(e, UD_KIND_CACHE);
        if (e->bf) conv_slot_zero<bf16>(e->slots_d, n, e->cg, e->stream);
        else conv_slot_zero<float>(e->slots_d, n, e->cg, e->stream);
    }
    if (e->cfg.joint_dim && e->rs.h) {
        Launch L_(e, UD_KIND_RNNT);
        rnnt_reset(e->rs, e->slots_d, n, e->rw, e->stream);
    }
    UD_CK(cudaGetLastError());
    return UD_OK;
}

ud_status ud_cache_read(ud_engine* e, ud_stream_id id, int layer, int kind, void* host_out) {
    if (!e || !host_out) return fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    UD_TRY(check_ids(e, 1, &id));
    if (layer < 0 || layer >= e->cfg.n_layers || kind < 0 || kind > 2)
        return fail(UD_ERR_INVALID_ARGUMENT, "layer or kind out of range");
    UD_CK(cudaSetDevice(e->device));
    const size_t kv = static_cast<size_t>(e->cfg.n_layers) * 2 * e->L * e->D * e->esz;
    const size_t cv = static_cast<size_t>(e->cfg.n_layers) * e->cg.conv_ring * e->D * e->esz;
    if (!e->gather_scratch) UD_TRY(dalloc_bytes(e, &e->gather_scratch, kv + cv));
    uint8_t* g = static_cast<uint8_t*>(e->gather_scratch);
    UD_TRY(ud_cache_gather(e, 1, &id, g, g + kv));
    UD_TRY(check_device_error(e));
    const size_t row = static_cast<size_t>(e->D) * e->esz;
    if (kind < 2)
        UD_CK(cudaMemcpyAsync(host_out, g + (static_cast<size_t>(layer) * 2 + kind) * e->L * row, e->L * row,
                              cudaMemcpyDeviceToHost, e->stream));
    else
        UD_CK(cudaMemcpyAsync(host_out, g + kv + static_cast<size_t>(layer) * e->cg.conv_ring * row,
                              e->cg.conv_ring * row, cudaMemcpyDeviceToHost, e->stream));
    UD_CK(cudaStreamSynchronize(e->stream));
    return UD_OK;
}

ud_status ud_stream_info(ud_engine* e, ud_stream_id id, int* cache_len, int* head, int* step) {
    if (!e) return fail(UD_ERR_INVALID_ARGUMENT, "NULL engine");
    UD_TRY(check_ids(e, 1, &id));
    const Slot& s = e->slots[id];
    if (cache_len) *cache_len = s.cache_len;
    if (head) *head = s.head;
    if (step) *step = s.step;
    return UD_OK;
}

ud_status ud_get_cuda_stream(ud_engine* e, void** stream_out) {
    if (!e || !stream_out) return fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    *stream_out = e->stream;
    return UD_OK;
}

ud_status ud_pool_info(ud_engine* e, int* free_pages, int* total_pages, int* elem_bytes) {
    if (!e) return fail(UD_ERR_INVALID_ARGUMENT, "NULL engine");
    if (free_pages) *free_pages = static_cast<int>(e->free_pages.size());
    if (total_pages) *total_pages = e->cg.n_pages;
    if (elem_bytes) *elem_bytes = e->esz;
    return UD_OK;
}

ud_status ud_get_config(ud_engine* e, ud_config* out) {
    if (!e || !out) return fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = e->cfg;
    return UD_OK;
}

ud_status ud_synchronize(ud_engine* e) {
    if (!e) return fail(UD_ERR_INVALID_ARGUMENT, "NULL engine");
    UD_CK(cudaSetDevice(e->device));
    UD_CK(cudaGetLastError());
    UD_TRY(drain_async(e));   // pipelined steps complete too
    return check_device_error(e);
}

ud_status ud_launch_count(ud_engine* e, int64_t* out) {
    if (!e || !out) return fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = e->launches;
    return UD_OK;
}

ud_status ud_debug_gemm(ud_engine* e, const void* A, const void* W, int M, int N, int K, const float* bias, int act,
                        float out_scale, const float* residual, float res_scale, void* Cout, int out_bf16) {
    if (!e || !A || !W || !Cout || M < 1 || N < 1 || K < 1) return fail(UD_ERR_INVALID_ARGUMENT, "bad argument");
    if (act < 0 || act > 2) return fail(UD_ERR_INVALID_ARGUMENT, "bad activation");
    UD_CK(cudaSetDevice(e->device));
    WeightMat wm;
    wm.p = const_cast<void*>(W);
    wm.N = N;
    wm.K = K;
    if (e->bf && tc_ok(N, K)) {
        if (!make_tma_bf16(wm.tma128, W, N, K, K, 128)) return fail(UD_ERR_CUDA, "tensor map failed");
        wm.has_tma = true;
        if (N % 256 == 0 && make_tma_bf16(wm.tma256, W, N, K, K, 256)) wm.has256 = true;
    }
    GemmEpilogue g;
    g.bias = bias;
    g.act = act;
    g.out_scale = out_scale;
    g.residual = residual;
    g.ldr = N;
    g.res_scale = res_scale;
    g.out = Cout;
    g.ldo = N;
    g.out_bf16 = out_bf16;
    UD_TRY(gemm(e, A, K, M, wm, g));
    UD_CK(cudaGetLastError());
    return check_device_error(e);
}

ud_status ud_debug_wait_probe(ud_engine* e, uint64_t limit_ns) {
    if (!e) return fail(UD_ERR_INVALID_ARGUMENT, "NULL engine");
    if (limit_ns > 10000000000ull) return fail(UD_ERR_INVALID_ARGUMENT, "limit above 10 s");
    UD_CK(cudaSetDevice(e->device));
    {
        Launch L_(e, UD_KIND_OTHER);
        test_wait_timeout(e->err_d, limit_ns, e->stream);
    }
    UD_CK(cudaGetLastError());
    return check_device_error(e);
}

ud_status ud_profile_enable(ud_engine* e, int enable) {
    if (!e) return fail(UD_ERR_INVALID_ARGUMENT, "NULL engine");
    UD_CK(cudaSetDevice(e->device));
    prof_flush(e);
    e->prof = enable != 0;
    for (int k = 0; k < UD_KIND_COUNT; ++k) {
        e->prof_ms[k] = 0.0;
        e->prof_n[k] = 0;
    }
    return UD_OK;
}

ud_status ud_graph_timers(ud_engine* e, int enable) {
    if (!e) return fail(UD_ERR_INVALID_ARGUMENT, "NULL engine");
    UD_CK(cudaSetDevice(e->device));
    if (enable && !e->timer_buf) UD_TRY(dalloc(e, &e->timer_buf, 2 * static_cast<size_t>(kTimerSlots)));
    e->timers = enable != 0;
    e->timer_last_kinds.clear();
    return UD_OK;
}

ud_status ud_graph_timers_read(ud_engine* e, int kind, double* ms, int* launches) {
    if (!e || !ms || !launches || kind < 0 || kind >= UD_KIND_COUNT) return fail(UD_ERR_INVALID_ARGUMENT, "bad argument");
    UD_CK(cudaSetDevice(e->device));
    *ms = 0.0;
    *launches = 0;
    if (!e->timer_buf || e->timer_last_kinds.empty()) return UD_OK;
    const int n = static_cast<int>(e->timer_last_kinds.size());
    std::vector<unsigned long long> h(2 * static_cast<size_t>(kTimerSlots));
    UD_CK(cudaStreamSynchronize(e->stream));
    UD_CK(cudaMemcpy(h.data(), e->timer_buf, sizeof(unsigned long long) * h.size(), cudaMemcpyDeviceToHost));
    double ns = 0.0;
    int counted = 0;
    for (int i = 0; i < n; ++i) {
        if (e->timer_last_kinds[i] != kind) continue;
        const unsigned long long t0 = h[i], t1 = h[kTimerSlots + i];
        if (t0 == ~0ull || t1 < t0) continue;   // a slot its kernel did not use (another path ran)
        ns += static_cast<double>(t1 - t0);
        ++counted;
    }
    *ms = ns * 1e-6;
    *launches = counted;
    return UD_OK;
}

ud_status ud_profile_read(ud_engine* e, int kind, double* ms_total, int64_t* launches) {
    if (!e || kind < 0 || kind >= UD_KIND_COUNT) return fail(UD_ERR_INVALID_ARGUMENT, "bad argument");
    UD_CK(cudaSetDevice(e->device));
    prof_flush(e);
    if (ms_total) *ms_total = e->prof_ms[kind];
    if (launches) *launches = e->prof_n[kind];
    return UD_OK;
}

}  // extern "C"
