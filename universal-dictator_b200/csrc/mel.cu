// Log-mel frontend: the B200 form of NemoMelFrontend / NemoMelStream (Sources/DictatorCore/Audio/NemoMel.swift),
// NeMo's FilterbankFeatures at inference (dither off, no normalisation):
//   preemphasis y[0] = x[0], y[n] = x[n] - 0.97 x[n-1]                               (NemoMel.swift:48-52)
//   centred STFT, n_fft 512, hop 160, 400-tap window at taps 56..455 of the frame     (:54-65)
//   power |X|^2 (magnitude, then squared), mel = fb . power, log(mel + 2^-24)        (:91-107)
//   frames t >= N / 160 are 0 (the last frame of an utterance)                        (:104-106)
// The reference evaluates the DFT as two matrix products against cos/sin tables (:86-97). Here one warp takes
// one frame: the 512 real samples become a 256-point complex sequence, transformed in registers and across the
// warp's lanes (decimation in frequency: three in-lane stages, five shuffle stages), unpacked into the 257 bins
// through shared memory; the mel projection visits only each filter's non-zero bins.
// Frames are independent, so any mix of utterances and live streams runs in one launch: a table of utterance
// segments (24 bytes each) describes them, and each warp finds its frame's segment by binary search.
//
// Live streams keep, on the host, the raw samples the next frames still need; each push stages
// [kept tail ; new samples] of every stream in one host-to-device copy and returns the frames whose windows are
// complete (NemoMelStream.push, :124-135); finish emits the rest with the right zero padding (:138-143).
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "ud.h"

namespace ud {
ud_status host_fail(ud_status s, const char* msg);
cudaStream_t engine_stream(ud_engine* e);
int engine_device(ud_engine* e);
int engine_num_sms(ud_engine* e);
}  // namespace ud

namespace {

using ud::host_fail;

constexpr int kFFT = 512, kHalf = 256, kBins = 257, kHop = 160, kWin = 400, kWinOff = 56;
constexpr int kMelWarps = 8;

// A run of consecutive frames of one utterance.
struct MelSeg {
    int64_t base;    // buffer index of the utterance's sample 0 (only samples its frames read are present)
    int32_t n;       // samples of the utterance that exist (the right edge)
    int32_t t0;      // first frame index of the run within the utterance
    int32_t valid;   // frames t >= valid are written as zeros
    int32_t f0;      // index of the run's first frame among all frames of the launch (runs in order)
    int32_t row0;    // output row of frame t0
    int32_t pad;
};

struct MelGeom {
    const float* window;    // [400]
    const float* tw_c;      // [257] cos(2 pi k / 512)
    const float* tw_s;      // [257] sin(2 pi k / 512)
    const int* fb_lo;       // [n_mels] first non-zero bin of each filter
    const int* fb_len;      // [n_mels] its non-zero span
    const int* fb_off;      // [n_mels] offset of the span's weights in fb_w
    const float* fb_w;
    int n_mels;
};

// Storage index of FFT point i in a warp's spectrum buffer: one pad word per 32 keeps both the lane-ordered
// stores and the bit-reversed reads of the unpacking free of bank conflicts.
__device__ __forceinline__ int zpad(int i) { return i + (i >> 5); }

__global__ void __launch_bounds__(kMelWarps * 32) mel_kernel(const float* __restrict__ audio,
                                                             const MelSeg* __restrict__ segs, int n_segs,
                                                             int n_frames, const MelGeom g, float* __restrict__ out) {
    constexpr int kZ = kHalf + kHalf / 32;
    __shared__ float re[kMelWarps][kZ], im[kMelWarps][kZ], pw[kMelWarps][kBins + 3];
    __shared__ float win[kWin], tc[kBins], ts[kBins];
    for (int i = threadIdx.x; i < kWin; i += blockDim.x) win[i] = g.window[i];
    for (int i = threadIdx.x; i < kBins; i += blockDim.x) {
        tc[i] = g.tw_c[i];
        ts[i] = g.tw_s[i];
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* zr = re[warp];
    float* zi = im[warp];
    float* P = pw[warp];
    // The 256-point FFT is decimation in frequency over i = lane + 32 j: the distances 128, 64 and 32 pair
    // values of one lane (registers), 16 .. 1 pair lanes (shuffles). W_N^n = exp(-2 pi i n / N) = tc - i ts at
    // table index n * 512 / N; each lane's twiddles depend only on the lane and are loaded once.
    float w1c[4], w1s[4], w2c[2], w2s[2], wxc[5], wxs[5];
#pragma unroll
    for (int j = 0; j < 4; ++j) { w1c[j] = tc[2 * (lane + 32 * j)]; w1s[j] = ts[2 * (lane + 32 * j)]; }  // W_256
#pragma unroll
    for (int j = 0; j < 2; ++j) { w2c[j] = tc[4 * (lane + 32 * j)]; w2s[j] = ts[4 * (lane + 32 * j)]; }  // W_128
    const float w3c = tc[8 * lane], w3s = ts[8 * lane];                                           // W_64^lane
#pragma unroll
    for (int st = 0; st < 5; ++st) {
        const int d = 16 >> st;
        const int k = (lane & (d - 1)) * (256 / d);                                               // W_2d^(lane mod d)
        wxc[st] = tc[k];
        wxs[st] = ts[k];
    }
    for (int fi = blockIdx.x * kMelWarps + warp; fi < n_frames; fi += gridDim.x * kMelWarps) {
        int lo = 0, hi = n_segs - 1;   // last run with f0 <= fi
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (segs[mid].f0 <= fi) lo = mid;
            else hi = mid - 1;
        }
        const MelSeg f = segs[lo];
        const int t = f.t0 + (fi - f.f0);
        float* orow = out + static_cast<size_t>(f.row0 + (fi - f.f0)) * g.n_mels;
        if (t >= f.valid) {
            for (int m = lane; m < g.n_mels; m += 32) orow[m] = 0.f;
            continue;
        }
        // z[i] = v[2i] + i v[2i+1], v = the windowed preemphasised samples at frame positions 0..511.
        const int64_t s0 = static_cast<int64_t>(t) * kHop - kWin / 2;   // utterance index of window tap 0
        float vr[8], vi[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = lane + 32 * j;
            float v[2];
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int pos = 2 * i + c;
                v[c] = 0.f;
                if (pos >= kWinOff && pos < kWinOff + kWin) {
                    const int64_t smp = s0 + (pos - kWinOff);
                    if (smp >= 0 && smp < f.n) {
                        const float x = audio[f.base + smp];
                        const float y = smp == 0 ? x : __fsub_rn(x, __fmul_rn(0.97f, audio[f.base + smp - 1]));
                        v[c] = __fmul_rn(y, win[pos - kWinOff]);
                    }
                }
            }
            vr[j] = v[0];
            vi[j] = v[1];
        }
        // Butterfly (a, b) -> (a + b, (a - b) W).
        auto bfly = [](float& ar, float& ai, float& br, float& bi, float c, float s) {
            const float dr = ar - br, di = ai - bi;
            ar += br;
            ai += bi;
            br = dr * c + di * s;
            bi = di * c - dr * s;
        };
#pragma unroll
        for (int j = 0; j < 4; ++j) bfly(vr[j], vi[j], vr[j + 4], vi[j + 4], w1c[j], w1s[j]);
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if ((j & 2) == 0) bfly(vr[j], vi[j], vr[j + 2], vi[j + 2], w2c[j & 1], w2s[j & 1]);
#pragma unroll
        for (int j = 0; j < 8; j += 2) bfly(vr[j], vi[j], vr[j + 1], vi[j + 1], w3c, w3s);
#pragma unroll
        for (int st = 0; st < 5; ++st) {
            const int d = 16 >> st;
            const bool upper = (lane & d) != 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float pr = __shfl_xor_sync(0xffffffffu, vr[j], d);
                const float pi = __shfl_xor_sync(0xffffffffu, vi[j], d);
                const float dr = pr - vr[j], di = pi - vi[j];
                const float sr = vr[j] + pr, si = vi[j] + pi;
                vr[j] = upper ? dr * wxc[st] + di * wxs[st] : sr;
                vi[j] = upper ? di * wxc[st] - dr * wxs[st] : si;
            }
        }
        // Point i now holds Z[bitrev8(i)].
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            zr[zpad(lane + 32 * j)] = vr[j];
            zi[zpad(lane + 32 * j)] = vi[j];
        }
        __syncwarp();
        // Real-input spectrum: X[k] = E[k] - i W^k D[k], E/D the even/odd parts of Z[k] and conj(Z[256-k]).
        for (int k = lane; k < kBins; k += 32) {
            const int ka = zpad(__brev(k & (kHalf - 1)) >> 24), kb = zpad(__brev((kHalf - k) & (kHalf - 1)) >> 24);
            const float Ar = zr[ka], Ai = zi[ka], Br = zr[kb], Bi = -zi[kb];
            const float Er = 0.5f * (Ar + Br), Ei = 0.5f * (Ai + Bi);
            const float Dr = 0.5f * (Ar - Br), Di = 0.5f * (Ai - Bi);
            const float c = tc[k], s = ts[k];
            const float Xr = Er + c * Di - s * Dr, Xi = Ei - c * Dr - s * Di;
            const float mag = sqrtf(__fadd_rn(__fmul_rn(Xr, Xr), __fmul_rn(Xi, Xi)));
            P[k] = __fmul_rn(mag, mag);
        }
        __syncwarp();
        for (int m = lane; m < g.n_mels; m += 32) {
            const int lo2 = g.fb_lo[m], len = g.fb_len[m];
            const float* w = g.fb_w + g.fb_off[m];
            float acc = 0.f;
            for (int j = 0; j < len; ++j) acc = fmaf(w[j], P[lo2 + j], acc);
            orow[m] = logf(acc + 5.9604644775390625e-8f);   // + 2^-24
        }
        __syncwarp();
    }
}

struct MelStream {
    bool open = false, finished = false;
    int64_t n = 0;          // samples received
    int64_t tail0 = 0;      // utterance index of tail[0]
    int frames = 0;         // frames emitted
    std::vector<float> tail;
};

}  // namespace

struct ud_mel {
    ud_engine* e = nullptr;
    int device = 0, num_sms = 148, n_mels = 0;
    cudaStream_t stream = nullptr;
    MelGeom g{};
    std::vector<void*> allocs;
    // per-call staging (grown on demand; the stream is synchronised before a buffer is replaced)
    float* samples_h = nullptr;
    float* samples_d = nullptr;
    size_t samples_cap = 0;
    MelSeg* segs_h = nullptr;
    MelSeg* segs_d = nullptr;
    size_t segs_cap = 0;
    float* mel_h = nullptr;
    float* mel_d = nullptr;
    size_t mel_cap = 0;   // rows
    cudaEvent_t staged = nullptr;   // recorded after the uploads of the last call
    std::vector<MelStream> streams;
    std::vector<int> free_ids;
};

namespace {

template <typename T>
ud_status dev_alloc(ud_mel* m, T** p, size_t count) {
    void* q = nullptr;
    if (cudaMalloc(&q, std::max<size_t>(count, 1) * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return host_fail(UD_ERR_OUT_OF_MEMORY, "cudaMalloc failed (mel)");
    }
    m->allocs.push_back(q);
    *p = static_cast<T*>(q);
    return UD_OK;
}

// Replaces a (host pinned, device) buffer pair by one of at least `need` elements.
template <typename T>
ud_status grow(ud_mel* m, T** h, T** d, size_t* cap, size_t need) {
    if (need <= *cap) return UD_OK;
    if (cudaStreamSynchronize(m->stream) != cudaSuccess) return host_fail(UD_ERR_CUDA, "stream synchronize failed");
    const size_t c = std::max(need, *cap * 2);
    if (*h) cudaFreeHost(*h);
    if (*d) {
        cudaFree(*d);
        m->allocs.erase(std::find(m->allocs.begin(), m->allocs.end(), static_cast<void*>(*d)));
    }
    *h = nullptr;
    *d = nullptr;
    *cap = 0;
    void* q = nullptr;
    if (cudaMallocHost(&q, c * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return host_fail(UD_ERR_OUT_OF_MEMORY, "cudaMallocHost failed (mel)");
    }
    *h = static_cast<T*>(q);
    ud_status s = dev_alloc(m, d, c);
    if (s != UD_OK) return s;
    *cap = c;
    return UD_OK;
}

void launch_frames(ud_mel* m, const float* audio_d, const MelSeg* segs_d, int n_segs, int n_frames, float* out_d) {
    if (n_frames <= 0) return;
    const int blocks = std::min((n_frames + kMelWarps - 1) / kMelWarps, m->num_sms * 8);
    mel_kernel<<<blocks, kMelWarps * 32, 0, m->stream>>>(audio_d, segs_d, n_segs, n_frames, m->g, out_d);
}

// Waits until the previous call's uploads have left the pinned staging buffers.
ud_status wait_staged(ud_mel* m) {
    if (cudaEventSynchronize(m->staged) != cudaSuccess) return host_fail(UD_ERR_CUDA, "event synchronize failed");
    return UD_OK;
}

}  // namespace

extern "C" {

ud_status ud_mel_create(ud_engine* e, const float* fb, int n_mels, const float* window, int max_streams,
                        ud_mel** out) {
    if (!e || !fb || !window || !out) return host_fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (n_mels < 1 || n_mels > 1024 || max_streams < 0)
        return host_fail(UD_ERR_INVALID_ARGUMENT, "n_mels or max_streams out of range");
    ud_mel* m = new ud_mel;
    m->e = e;
    m->device = ud::engine_device(e);
    m->stream = ud::engine_stream(e);
    m->num_sms = ud::engine_num_sms(e);
    m->n_mels = n_mels;
    auto bail = [&](ud_status s) {
        ud_mel_destroy(m);
        return s;
    };
    if (cudaSetDevice(m->device) != cudaSuccess) return bail(host_fail(UD_ERR_CUDA, "cudaSetDevice failed"));
    // Filters as non-zero spans (the full row when a filter is zero everywhere: it then sums zeros).
    std::vector<int> lo(n_mels), len(n_mels), off(n_mels);
    std::vector<float> w;
    for (int r = 0; r < n_mels; ++r) {
        const float* row = fb + static_cast<size_t>(r) * kBins;
        int a = 0, b = kBins - 1;
        while (a < kBins && row[a] == 0.f) ++a;
        while (b >= a && row[b] == 0.f) --b;
        if (a > b) { a = 0; b = 0; }
        lo[r] = a;
        len[r] = b - a + 1;
        off[r] = static_cast<int>(w.size());
        w.insert(w.end(), row + a, row + b + 1);
    }
    std::vector<float> c(kBins), s(kBins);
    for (int k = 0; k < kBins; ++k) {
        const double th = 2.0 * 3.14159265358979323846 * k / kFFT;
        c[k] = static_cast<float>(std::cos(th));
        s[k] = static_cast<float>(std::sin(th));
    }
    float *win_d, *c_d, *s_d, *w_d;
    int *lo_d, *len_d, *off_d;
    ud_status st;
    if ((st = dev_alloc(m, &win_d, kWin)) != UD_OK || (st = dev_alloc(m, &c_d, kBins)) != UD_OK ||
        (st = dev_alloc(m, &s_d, kBins)) != UD_OK || (st = dev_alloc(m, &w_d, w.size())) != UD_OK ||
        (st = dev_alloc(m, &lo_d, n_mels)) != UD_OK || (st = dev_alloc(m, &len_d, n_mels)) != UD_OK ||
        (st = dev_alloc(m, &off_d, n_mels)) != UD_OK)
        return bail(st);
    bool ok = cudaMemcpyAsync(win_d, window, sizeof(float) * kWin, cudaMemcpyHostToDevice, m->stream) == cudaSuccess;
    ok = ok && cudaMemcpyAsync(c_d, c.data(), sizeof(float) * kBins, cudaMemcpyHostToDevice, m->stream) == cudaSuccess;
    ok = ok && cudaMemcpyAsync(s_d, s.data(), sizeof(float) * kBins, cudaMemcpyHostToDevice, m->stream) == cudaSuccess;
    ok = ok && cudaMemcpyAsync(w_d, w.data(), sizeof(float) * w.size(), cudaMemcpyHostToDevice, m->stream) == cudaSuccess;
    ok = ok && cudaMemcpyAsync(lo_d, lo.data(), sizeof(int) * n_mels, cudaMemcpyHostToDevice, m->stream) == cudaSuccess;
    ok = ok && cudaMemcpyAsync(len_d, len.data(), sizeof(int) * n_mels, cudaMemcpyHostToDevice, m->stream) == cudaSuccess;
    ok = ok && cudaMemcpyAsync(off_d, off.data(), sizeof(int) * n_mels, cudaMemcpyHostToDevice, m->stream) == cudaSuccess;
    ok = ok && cudaStreamSynchronize(m->stream) == cudaSuccess;
    ok = ok && cudaEventCreateWithFlags(&m->staged, cudaEventDisableTiming) == cudaSuccess;
    if (!ok) return bail(host_fail(UD_ERR_CUDA, "mel frontend upload failed"));
    m->g = MelGeom{win_d, c_d, s_d, lo_d, len_d, off_d, w_d, n_mels};
    m->streams.resize(static_cast<size_t>(max_streams));
    for (int i = max_streams - 1; i >= 0; --i) m->free_ids.push_back(i);
    *out = m;
    return UD_OK;
}

ud_status ud_mel_destroy(ud_mel* m) {
    if (!m) return UD_OK;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (void* p : m->allocs) cudaFree(p);
    if (m->samples_h) cudaFreeHost(m->samples_h);
    if (m->segs_h) cudaFreeHost(m->segs_h);
    if (m->mel_h) cudaFreeHost(m->mel_h);
    if (m->staged) cudaEventDestroy(m->staged);
    delete m;
    return UD_OK;
}

ud_status ud_mel_features_device(ud_mel* m, int n, const float* audio_dev, const int64_t* sample_off,
                                 const int* n_samples, float* mel_dev, const int64_t* row_off) {
    if (!m || n < 0 || (n > 0 && (!audio_dev || !sample_off || !n_samples || !mel_dev || !row_off)))
        return host_fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    size_t total = 0;
    for (int i = 0; i < n; ++i) {
        if (n_samples[i] < 0 || sample_off[i] < 0 || row_off[i] < 0)
            return host_fail(UD_ERR_INVALID_ARGUMENT, "negative length or offset");
        total += static_cast<size_t>(n_samples[i] / kHop + 1);
    }
    if (total > static_cast<size_t>(INT32_MAX)) return host_fail(UD_ERR_INVALID_ARGUMENT, "too many frames");
    if (cudaSetDevice(m->device) != cudaSuccess) return host_fail(UD_ERR_CUDA, "cudaSetDevice failed");
    ud_status st = wait_staged(m);
    if (st != UD_OK) return st;
    if ((st = grow(m, &m->segs_h, &m->segs_d, &m->segs_cap, static_cast<size_t>(n))) != UD_OK) return st;
    int k = 0, f0 = 0;
    for (int i = 0; i < n; ++i) {
        const int T = n_samples[i] / kHop + 1;
        if (row_off[i] + T > INT32_MAX) return host_fail(UD_ERR_INVALID_ARGUMENT, "output row out of range");
        m->segs_h[k++] = MelSeg{sample_off[i], n_samples[i], 0, n_samples[i] / kHop, f0, static_cast<int32_t>(row_off[i]), 0};
        f0 += T;
    }
    if (k > 0 && cudaMemcpyAsync(m->segs_d, m->segs_h, sizeof(MelSeg) * k, cudaMemcpyHostToDevice, m->stream) != cudaSuccess)
        return host_fail(UD_ERR_CUDA, "segment table upload failed");
    cudaEventRecord(m->staged, m->stream);
    launch_frames(m, audio_dev, m->segs_d, k, f0, mel_dev);
    if (cudaGetLastError() != cudaSuccess) return host_fail(UD_ERR_CUDA, "mel kernel launch failed");
    return UD_OK;
}

ud_status ud_mel_stream_open(ud_mel* m, int* id) {
    if (!m || !id) return host_fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (m->free_ids.empty()) return host_fail(UD_ERR_POOL_EXHAUSTED, "no free mel stream");
    const int i = m->free_ids.back();
    m->free_ids.pop_back();
    m->streams[i] = MelStream();
    m->streams[i].open = true;
    *id = i;
    return UD_OK;
}

ud_status ud_mel_stream_close(ud_mel* m, int id) {
    if (!m || id < 0 || id >= static_cast<int>(m->streams.size()) || !m->streams[id].open)
        return host_fail(UD_ERR_NO_STREAM, "unknown mel stream");
    m->streams[id] = MelStream();
    m->free_ids.push_back(id);
    return UD_OK;
}

ud_status ud_mel_push_batch(ud_mel* m, int n, const int* ids, const float* const* audio, const int* n_samples,
                            const int* finish, float* mel_out, int cap_frames, int* frames_out) {
    if (!m || n < 0 || (n > 0 && (!ids || !audio || !n_samples || !mel_out || !frames_out)))
        return host_fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (cap_frames < 0) return host_fail(UD_ERR_INVALID_ARGUMENT, "negative capacity");
    // Validate everything before any state changes.
    for (int i = 0; i < n; ++i) {
        const int id = ids[i];
        if (id < 0 || id >= static_cast<int>(m->streams.size()) || !m->streams[id].open)
            return host_fail(UD_ERR_NO_STREAM, "unknown mel stream");
        for (int j = 0; j < i; ++j)
            if (ids[j] == id) return host_fail(UD_ERR_INVALID_ARGUMENT, "a mel stream appears twice in one batch");
        const MelStream& s = m->streams[id];
        if (s.finished) return host_fail(UD_ERR_INVALID_ARGUMENT, "samples pushed after finish");
        if (n_samples[i] < 0 || (n_samples[i] > 0 && !audio[i]))
            return host_fail(UD_ERR_INVALID_ARGUMENT, "bad sample count or pointer");
        const int64_t nn = s.n + n_samples[i];
        const int64_t end = (finish && finish[i]) ? nn / kHop + 1 : (nn >= kWin / 2 ? (nn - kWin / 2) / kHop + 1 : 0);
        if (end > INT32_MAX / 2) return host_fail(UD_ERR_INVALID_ARGUMENT, "stream too long");
        if (end - s.frames > cap_frames) return host_fail(UD_ERR_INVALID_ARGUMENT, "mel_out too small for the frames");
    }
    if (cudaSetDevice(m->device) != cudaSuccess) return host_fail(UD_ERR_CUDA, "cudaSetDevice failed");
    ud_status st = wait_staged(m);
    if (st != UD_OK) return st;
    // Plan: append, then stage each stream's needed samples [first sample of its next frame - 1, end).
    std::vector<int64_t> first(n), stage_off(n);
    std::vector<int> end(n), valid(n);
    size_t samples = 0, total = 0;
    for (int i = 0; i < n; ++i) {
        MelStream& s = m->streams[ids[i]];
        s.tail.insert(s.tail.end(), audio[i], audio[i] + n_samples[i]);
        s.n += n_samples[i];
        const bool fin = finish && finish[i];
        end[i] = fin ? static_cast<int>(s.n / kHop + 1)
                     : (s.n >= kWin / 2 ? static_cast<int>((s.n - kWin / 2) / kHop + 1) : 0);
        valid[i] = fin ? static_cast<int>(s.n / kHop) : INT32_MAX;
        first[i] = std::max<int64_t>(s.tail0, static_cast<int64_t>(s.frames) * kHop - kWin / 2 - 1);
        stage_off[i] = static_cast<int64_t>(samples);
        samples += static_cast<size_t>(s.n - first[i]);
        total += static_cast<size_t>(std::max(0, end[i] - s.frames));
        frames_out[i] = std::max(0, end[i] - s.frames);
    }
    if ((st = grow(m, &m->samples_h, &m->samples_d, &m->samples_cap, samples)) != UD_OK) return st;
    if ((st = grow(m, &m->segs_h, &m->segs_d, &m->segs_cap, static_cast<size_t>(n))) != UD_OK) return st;
    if ((st = grow(m, &m->mel_h, &m->mel_d, &m->mel_cap, total * m->n_mels)) != UD_OK) return st;
    int k = 0, f0 = 0;
    for (int i = 0; i < n; ++i) {
        MelStream& s = m->streams[ids[i]];
        const int64_t cnt = s.n - first[i];
        if (cnt > 0) std::memcpy(m->samples_h + stage_off[i], s.tail.data() + (first[i] - s.tail0), sizeof(float) * cnt);
        const int nf = std::max(0, end[i] - s.frames);
        if (nf == 0) continue;
        m->segs_h[k++] = MelSeg{stage_off[i] - first[i], static_cast<int32_t>(s.n), s.frames, valid[i], f0, f0, 0};
        f0 += nf;
    }
    if (total > 0) {
        bool ok = samples == 0 || cudaMemcpyAsync(m->samples_d, m->samples_h, sizeof(float) * samples,
                                                  cudaMemcpyHostToDevice, m->stream) == cudaSuccess;
        ok = ok && cudaMemcpyAsync(m->segs_d, m->segs_h, sizeof(MelSeg) * k, cudaMemcpyHostToDevice,
                                   m->stream) == cudaSuccess;
        if (!ok) return host_fail(UD_ERR_CUDA, "mel staging upload failed");
        cudaEventRecord(m->staged, m->stream);
        launch_frames(m, m->samples_d, m->segs_d, k, static_cast<int>(total), m->mel_d);
        if (cudaGetLastError() != cudaSuccess) return host_fail(UD_ERR_CUDA, "mel kernel launch failed");
        if (cudaMemcpyAsync(m->mel_h, m->mel_d, sizeof(float) * total * m->n_mels, cudaMemcpyDeviceToHost,
                            m->stream) != cudaSuccess ||
            cudaStreamSynchronize(m->stream) != cudaSuccess)
            return host_fail(UD_ERR_CUDA, "mel readback failed");
    }
    size_t row = 0;
    for (int i = 0; i < n; ++i) {
        MelStream& s = m->streams[ids[i]];
        const int nf = std::max(0, end[i] - s.frames);
        if (nf > 0)
            std::memcpy(mel_out + static_cast<size_t>(i) * cap_frames * m->n_mels, m->mel_h + row * m->n_mels,
                        sizeof(float) * nf * m->n_mels);
        row += static_cast<size_t>(nf);
        s.frames = std::max(s.frames, end[i]);
        if (finish && finish[i]) s.finished = true;
        // Keep from the raw sample before the next frame's first window tap.
        const int64_t keep = std::max<int64_t>(s.tail0, static_cast<int64_t>(s.frames) * kHop - kWin / 2 - 1);
        if (keep > s.tail0) {
            s.tail.erase(s.tail.begin(), s.tail.begin() + (keep - s.tail0));
            s.tail0 = keep;
        }
    }
    return UD_OK;
}

ud_status ud_mel_features(ud_mel* m, const float* audio, int n_samples, float* mel_out, int cap_frames,
                          int* frames_out) {
    if (!m || (n_samples > 0 && !audio) || !mel_out || !frames_out)
        return host_fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (n_samples < 0) return host_fail(UD_ERR_INVALID_ARGUMENT, "negative sample count");
    const int T = n_samples / kHop + 1;
    if (T > cap_frames) return host_fail(UD_ERR_INVALID_ARGUMENT, "mel_out too small for the frames");
    // One temporary stream holding the whole utterance, finished at once.
    if (m->free_ids.empty()) {
        m->streams.emplace_back();
        m->free_ids.push_back(static_cast<int>(m->streams.size()) - 1);
    }
    int id;
    ud_status st = ud_mel_stream_open(m, &id);
    if (st != UD_OK) return st;
    const int fin = 1;
    st = ud_mel_push_batch(m, 1, &id, &audio, &n_samples, &fin, mel_out, cap_frames, frames_out);
    ud_mel_stream_close(m, id);
    return st;
}

}  // extern "C"
