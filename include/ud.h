/*
 * ud.h — C ABI of the B200 streaming FastConformer engine (libud.so).
 *
 * This is the drop-in boundary for the reference's encoder protocol
 *   public protocol NemotronEncoder: AnyObject {
 *       var schedule: NemotronSchedule { get }
 *       func step(mel: UnsafeBufferPointer<Float>, nRows: Int, validRows: Int, keepAll: Bool) throws
 *           -> (proj: [Float], frames: Int)
 *   }                                   (Sources/DictatorCore/Nemotron/NemotronStreamer.swift:6-12)
 * whose GPU implementation is MetalNemotronEncoder (Sources/DictatorEngine/Models/Nemotron.swift:51-91)
 * over FastConformerEncoder.encodeStreamStep (Sources/DictatorEngine/Models/FastConformer.swift:441-480).
 *
 * Plain C types only; no PyTorch. Every call returns ud_status (UD_OK = 0) and never aborts; the text
 * of the last error on the calling thread is available from ud_last_error(). An engine is bound to one
 * CUDA device and one CUDA stream. Calls on one engine must be serialised by the caller, as the
 * reference drives one stream from one serial queue (Sources/DictatorCore/API/Dictation.swift:301).
 * Different engines (for example one per GPU) may be used from different threads.
 */
#ifndef UD_H
#define UD_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define UD_ABI_VERSION 1

#if defined(__GNUC__)
#define UD_API __attribute__((visibility("default")))
#else
#define UD_API
#endif

typedef enum ud_status {
    UD_OK = 0,
    UD_ERR_INVALID_ARGUMENT = 1, /* a size, pointer or id out of range                              */
    UD_ERR_CUDA = 2,             /* a CUDA runtime/driver call failed                               */
    UD_ERR_OUT_OF_MEMORY = 3,    /* device or pinned host allocation failed                         */
    UD_ERR_NO_STREAM = 4,        /* unknown or closed stream id                                     */
    UD_ERR_POOL_EXHAUSTED = 5,   /* no free stream slot or cache page                               */
    UD_ERR_WEIGHTS = 6,          /* missing, duplicate or mis-shaped weight tensor                  */
    UD_ERR_NOT_READY = 7,        /* weights not loaded yet                                          */
    UD_ERR_DEVICE_TIMEOUT = 8,   /* a bounded device-side wait expired (the kernel returned early)  */
    UD_ERR_IO = 9,               /* file could not be read or parsed                                */
    UD_ERR_UNSUPPORTED = 10      /* configuration not supported by this build                       */
} ud_status;

typedef enum ud_dtype {
    UD_DTYPE_F32 = 0,  /* weights, activations and caches in fp32 (FFMA GEMMs)                       */
    UD_DTYPE_BF16 = 1  /* bf16 weights/activations/caches, fp32 accumulation, LN and softmax (tcgen05) */
} ud_dtype;

/* Static model + engine configuration (FastConformerConfig, FastConformer.swift:5-38, plus the
 * RNN-T head of RNNTDecoder, Sources/DictatorCore/Decoding/RNNT.swift:7-18). */
typedef struct ud_config {
    int n_layers;         /* 24                                                                      */
    int d_model;          /* 1024 (this build: 1024)                                                 */
    int n_heads;          /* 8    (head dim must be 128)                                             */
    int ff_dim;           /* 4096                                                                    */
    int conv_kernel;      /* 9    (causal depthwise; cache of conv_kernel-1 frames)                  */
    int left_context;     /* 70   (attention left context L of [L, R])                               */
    int sub_channels;     /* 256; 0 = no subsampling: steps take encoder frames instead of mel rows  */
    int mel_bins;         /* 128                                                                     */
    int joint_dim;        /* 640; 0 = no joint projection / RNN-T head                               */
    int vocab;            /* 1025 (1024 ids + blank; blank = vocab-1)                                */
    int pred_layers;      /* LSTM layers of the prediction net                                       */
    int pred_hidden;      /* 640                                                                     */
    int max_symbols;      /* greedy symbols per frame, 10                                            */
    int dtype;            /* ud_dtype                                                                */
    int max_streams;      /* concurrent stream slots                                                 */
    int max_batch;        /* streams per batched step                                                */
    int max_chunk_frames; /* largest T (encoder frames per step) any step may produce, <= 32         */
    int page_frames;      /* frames per cache page (16)                                              */
    int n_pages;          /* page pool size; 0 = enough for every slot                               */
} ud_config;

typedef struct ud_engine ud_engine;
typedef int32_t ud_stream_id;

/* One weight tensor in checkpoint naming and layout (docs/specs/nemotron.md section 8), fp32 host data. */
typedef struct ud_weight {
    const char* name;
    const float* data;
    int ndim;
    int64_t shape[4];
} ud_weight;

/* Nemotron defaults: 24 layers, d 1024, 8x128 heads, ff 4096, k 9, L 70, subsampling 256, joint 640,
 * vocab 1025, 1 LSTM layer of 640, bf16, 64 slots, batch 64, 16 frames per chunk, 16-frame pages. */
UD_API void ud_config_default(ud_config* cfg);

UD_API ud_status ud_init(const ud_config* cfg, int device, ud_engine** out);
UD_API ud_status ud_shutdown(ud_engine* e);

/* Copies (and converts) every tensor the configuration needs; all must be present with checkpoint
 * shapes. Replaces NemotronModel.init's weight loading (Sources/DictatorEngine/Models/Nemotron.swift:35-46). */
UD_API ud_status ud_load_weights(ud_engine* e, const ud_weight* table, int n);
/* Same from a safetensors file with F32/F16/BF16 tensors (Sources/DictatorEngine/Core/SafeTensors.swift). */
UD_API ud_status ud_load_safetensors(ud_engine* e, const char* path);

/* A stream = the caches and decoder state one NemotronEncoder object owns (zeroed on open). */
UD_API ud_status ud_stream_open(ud_engine* e, int lookahead, ud_stream_id* out);
UD_API ud_status ud_stream_close(ud_engine* e, ud_stream_id id);   /* evicts: frees its pages and slot */

/* The protocol call, one stream: mel [n_rows, mel_bins] fp32 host rows (pre-encode cache rows
 * included), the first valid_rows real. Writes proj_out [frames, joint_dim] fp32 host (room for
 * max_chunk_frames rows) and *frames_out = keep_all ? validT : min(validT, lookahead+1)
 * (Nemotron.swift:74-91). Synchronous. With sub_channels == 0 the input is encoder frames
 * [n_rows, d_model] and the output is the last layer's output [n_rows, d_model]. */
UD_API ud_status ud_stream_step(ud_engine* e, ud_stream_id id, const float* mel, int n_rows, int valid_rows,
                         int keep_all, float* proj_out, int* frames_out);

/* Batched protocol calls over n distinct streams (one encoder pass for all of them), host buffers.
 * mel[i] points at stream i's rows. proj_out: n * max_chunk_frames * joint_dim floats, stream i at
 * proj_out + i*max_chunk_frames*joint_dim (may be NULL when tokens are requested: the projections are then
 * not copied out). If tokens_out is not NULL the RNN-T greedy decoder
 * (RNNT.swift:127-151) also runs on the kept frames with each stream's carried state:
 * tokens_out holds n * max_chunk_frames * max_symbols ids, stream i at offset
 * i*max_chunk_frames*max_symbols, and n_tokens_out[i] their count. Synchronous. */
UD_API ud_status ud_step_batch(ud_engine* e, int n, const ud_stream_id* ids, const float* const* mel,
                        const int* n_rows, const int* valid_rows, const int* keep_all,
                        float* proj_out, int* frames_out, int32_t* tokens_out, int* n_tokens_out);

/* Pipelined form of ud_step_batch (no reference counterpart: a serving loop's overlap of host copies with
 * compute). Same arguments and results; the call enqueues the step's input copy, encoder pass and output copy
 * and returns without waiting for them. The input copy runs on a copy stream of its own while the previous step
 * computes, and the output copy on another while the next one computes (two staging buffers alternate). On return the
 * PREVIOUS asynchronous step is complete: its outputs are in its caller's buffers and its input rows may be
 * reused. This step's host buffers must stay untouched until the next ud_step_batch_async or ud_step_sync
 * returns. frames_out is filled on return. The copies are DMA only from pinned (page-locked) host memory
 * given as one buffer with a fixed stride between streams; other inputs are gathered through a pinned staging
 * buffer first. Device errors of a step are reported by the call that completes it. Every other entry point
 * that runs a step waits for outstanding asynchronous steps first. */
UD_API ud_status ud_step_batch_async(ud_engine* e, int n, const ud_stream_id* ids, const float* const* mel,
                              const int* n_rows, const int* valid_rows, const int* keep_all,
                              float* proj_out, int* frames_out, int32_t* tokens_out, int* n_tokens_out);

/* Waits until every asynchronous step is complete (outputs in place); reports a device error of the last one. */
UD_API ud_status ud_step_sync(ud_engine* e);

/* Same with device-resident input and outputs, asynchronous on the engine's CUDA stream:
 * mel_dev [n, rows_stride, mel_bins] fp32 (stream i's rows at i*rows_stride), proj_dev
 * [n, max_chunk_frames, joint_dim], tokens_dev / n_tokens_dev as above or NULL. frames_out (host)
 * is known before the kernels run and is filled on return. */
UD_API ud_status ud_step_batch_device(ud_engine* e, int n, const ud_stream_id* ids, const float* mel_dev,
                               int rows_stride, const int* n_rows, const int* valid_rows,
                               const int* keep_all, float* proj_dev, int* frames_out,
                               int32_t* tokens_dev, int* n_tokens_dev);

/* RNN-T greedy decode of projected frames f [frames, joint_dim] (fp32 host) with the stream's carried
 * decoder state (RNNT.swift:127-151). tokens_out has room for frames*max_symbols ids. */
UD_API ud_status ud_rnnt_decode(ud_engine* e, ud_stream_id id, const float* f, int frames, int32_t* tokens_out,
                         int* n_tokens_out);

/* Allocation-free variant of ud_rnnt_decode (no reference counterpart: the reference's decoder allocates its
 * tensors per call). Same arguments, results and carried decoder state, but the call's scratch (the frames, the
 * batch entry, the token buffer and count) lives in one fixed 256 KiB block of the library's static device
 * memory, and the call makes no cudaMalloc, cudaFree or host heap allocation. It is for callers that must not
 * allocate: a real-time audio thread, where an allocation can take a lock or wait for the device to go idle and
 * so miss the buffer deadline, and processes whose device memory is already fully reserved by another
 * allocator, where a new cudaMalloc fails.
 * Limit: 256 + 4*frames*max_symbols (rounded up to 256) + 4*frames*joint_dim <= 262144 bytes (100 frames at
 * joint_dim 640 and max_symbols 10); larger calls return UD_ERR_INVALID_ARGUMENT.
 * The block is shared by every engine and thread on a device: overlapping calls on one device race, and the
 * caller must serialize them. The first call on each device resolves the block's address
 * (cudaGetSymbolAddress) and must come before any stream capture on that device. The address is forgotten when
 * the last engine on the device shuts down, so a device reset (cudaDeviceReset) is safe only while no engine is
 * alive on that device. A bounded device wait that expires returns UD_ERR_DEVICE_TIMEOUT (the tokens are then
 * incomplete) and clears the device error word. The per-kernel profiler (ud_profile_enable) does not time this
 * call: its event bookkeeping allocates. Rejections return the status and clear the message that ud_last_error
 * reports. */
UD_API ud_status ud_rnnt_decode_static(ud_engine* e, ud_stream_id id, const float* f, int frames,
                                       int32_t* tokens_out, int* n_tokens_out);

/* Cache operations on the paged per-stream rings (the reference's cache roll, FastConformer.swift:464-477).
 * kind: 0 = K (projected keys), 1 = V (projected values), 2 = conv (depthwise-conv inputs).
 * Rows are in the engine dtype (bf16 or fp32), d_model wide, device pointers.
 *   append: kv_rows [n, n_layers, 2, k, d]; conv_rows [n, n_layers, k, d] (either may be NULL);
 *           writes the k frames after each stream's head (allocating pages as needed).
 *   roll:   head += k, cacheLen = min(cacheLen + k, L); frees pages that left the window (metadata).
 *   gather: kv_out [n, n_layers, 2, L, d] = each stream's window (unfilled rows zero);
 *           conv_out [n, n_layers, conv_kernel-1, d] (either may be NULL).
 *   evict:  close and reopen the stream (fresh zero caches, same id).
 * append/gather are asynchronous on the engine stream; use ud_synchronize before reading results. */
UD_API ud_status ud_cache_append(ud_engine* e, int n, const ud_stream_id* ids, int k, const void* kv_rows,
                          const void* conv_rows);
UD_API ud_status ud_cache_roll(ud_engine* e, int n, const ud_stream_id* ids, int k);
UD_API ud_status ud_cache_gather(ud_engine* e, int n, const ud_stream_id* ids, void* kv_out, void* conv_out);
UD_API ud_status ud_cache_evict(ud_engine* e, int n, const ud_stream_id* ids);
/* One stream's window of one layer and kind, copied to host: K/V [L, d], conv [conv_kernel-1, d]. */
UD_API ud_status ud_cache_read(ud_engine* e, ud_stream_id id, int layer, int kind, void* host_out);
/* cacheLen and absolute head frame of a stream. */
UD_API ud_status ud_stream_info(ud_engine* e, ud_stream_id id, int* cache_len, int* head, int* step);

/* Engine facts: the CUDA stream (cudaStream_t) work is issued on, free pages, element size. */
UD_API ud_status ud_get_cuda_stream(ud_engine* e, void** stream_out);
UD_API ud_status ud_pool_info(ud_engine* e, int* free_pages, int* total_pages, int* elem_bytes);
/* Waits for the engine's work, pipelined steps (ud_step_batch_async) included; reports a device error. */
UD_API ud_status ud_synchronize(ud_engine* e);
/* Number of this library's kernels launched on the engine since init (counts graph replays' kernels). */
UD_API ud_status ud_launch_count(ud_engine* e, int64_t* out);

/* Per-kernel-class timing (CUDA events around each launch on the engine stream). Off by default; enabling
 * it clears the totals. ud_profile_read synchronises and returns the summed device time and launch count
 * of one class. Used outside timed regions to attribute a step's time to its kernels. */
typedef enum ud_kernel_kind {
    UD_KIND_GEMM_TC = 0,    /* 1-CTA tcgen05 GEMM                              */
    UD_KIND_GEMM_SIMT = 1,  /* few-row / fp32 FFMA GEMM                         */
    UD_KIND_ATTENTION = 2,  /* rel-pos attention + K/V append                   */
    UD_KIND_CONV = 3,       /* conv module (GLU, depthwise, LN, SiLU, ring)     */
    UD_KIND_NORM = 4,       /* LayerNorm                                        */
    UD_KIND_SUBSAMPLE = 5,  /* subsampling convs, row select / pack             */
    UD_KIND_RNNT = 6,       /* RNN-T greedy                                     */
    UD_KIND_CACHE = 7,      /* cache append / gather / reset                    */
    UD_KIND_OTHER = 8,
    UD_KIND_GEMM_TC2 = 9,   /* 2-CTA (cta_group::2) tcgen05 GEMM, M >= 256     */
    UD_KIND_COUNT = 10
} ud_kernel_kind;
UD_API ud_status ud_profile_enable(ud_engine* e, int enable);
UD_API ud_status ud_profile_read(ud_engine* e, int kind, double* ms_total, int64_t* launches);

/* Graph-mode kernel timers. With enable != 0, the following steps' 2-CTA tcgen05 GEMM, TMA attention, LayerNorm
 * and conv-module launches each record, in global-timer nanoseconds, when their first CTA passed the
 * grid-dependency wait and when their last CTA's work ended; steps run with the timers on are captured in graphs
 * of their own, so the step's CUDA graph and programmatic dependent launch stay as in normal operation.
 * ud_graph_timers_read synchronises and returns, for the last step and one ud_kernel_kind (UD_KIND_GEMM_TC2,
 * UD_KIND_ATTENTION, UD_KIND_NORM or UD_KIND_CONV), the sum over its launches of (last end - first start) in
 * milliseconds and the number of launches. When the layer stack runs as two halves on two streams, the halves'
 * launches overlap and the sum counts both. */
UD_API ud_status ud_graph_timers(ud_engine* e, int enable);
UD_API ud_status ud_graph_timers_read(ud_engine* e, int kind, double* ms, int* launches);

/* Kernel-level test hook (the reference's GemmTests.swift contract, Step.gemm in Core/Kernels.swift:79-113):
 * C = out_scale * act(A . W^T + bias) + res_scale * R, device pointers, A [M,K] and W [N,K] in the
 * engine dtype, C fp32 [M,N] (or bf16 if out_bf16), act 0 none / 1 relu / 2 silu, R fp32 or NULL. */
UD_API ud_status ud_debug_gemm(ud_engine* e, const void* A, const void* W, int M, int N, int K, const float* bias,
                        int act, float out_scale, const float* residual, float res_scale, void* C, int out_bf16);

/* Failure-detection probe: launches a kernel that waits on a device flag nothing sets, with the same bounded
 * wait the pipelined kernels use; it gives up after limit_ns, and the call returns UD_ERR_DEVICE_TIMEOUT
 * with the engine still usable. */
UD_API ud_status ud_debug_wait_probe(ud_engine* e, uint64_t limit_ns);

/* The configuration the engine was created with. */
UD_API ud_status ud_get_config(ud_engine* e, ud_config* out);

/* ---- Log-mel frontend (NemoMelFrontend / NemoMelStream, Sources/DictatorCore/Audio/NemoMel.swift:10-161)
 *
 * NeMo's FilterbankFeatures at inference on the engine's device and CUDA stream: preemphasis 0.97, centred
 * STFT (n_fft 512, hop 160, the 400-tap window at taps 56..455), power, mel filterbank, log(x + 2^-24); frames
 * at or beyond n_samples / 160 are 0. fb [n_mels, 257] is the checkpoint's preprocessor.featurizer.fb and
 * window [400] its preprocessor.featurizer.window (NemoMelFrontend.init, :22-39). max_streams live streams can
 * be open at once. Output rows are time-major [frames, n_mels] fp32, the encoder's mel input. */
typedef struct ud_mel ud_mel;
UD_API ud_status ud_mel_create(ud_engine* e, const float* fb, int n_mels, const float* window, int max_streams,
                               ud_mel** out);
UD_API ud_status ud_mel_destroy(ud_mel* m);
/* Full utterance (NemoMelFrontend.features, :45-66): n_samples / 160 + 1 frames into mel_out (capacity
 * cap_frames rows), the last one 0; *frames_out = their count. */
UD_API ud_status ud_mel_features(ud_mel* m, const float* audio, int n_samples, float* mel_out, int cap_frames,
                                 int* frames_out);
/* Device-resident batch of n utterances, asynchronous on the engine stream: utterance i is n_samples[i] samples
 * at audio_dev + sample_off[i]; its n_samples[i] / 160 + 1 frames go to rows [row_off[i], ...) of mel_dev. */
UD_API ud_status ud_mel_features_device(ud_mel* m, int n, const float* audio_dev, const int64_t* sample_off,
                                        const int* n_samples, float* mel_dev, const int64_t* row_off);
/* Live streams (NemoMelStream, :110-161): push samples in any sizes; a frame is returned once its window is
 * complete (sample 160 t + 199 has arrived); finish != 0 ends the stream and returns the remaining frames with
 * the right zero padding and the zeroed last frame, so the frames equal ud_mel_features of the whole stream.
 * Stream i's new frames go to mel_out + i * cap_frames * n_mels, their count to frames_out[i]. */
UD_API ud_status ud_mel_stream_open(ud_mel* m, int* id);
UD_API ud_status ud_mel_stream_close(ud_mel* m, int id);
UD_API ud_status ud_mel_push_batch(ud_mel* m, int n, const int* ids, const float* const* audio, const int* n_samples,
                                   const int* finish, float* mel_out, int cap_frames, int* frames_out);

/* ---- Host-side batched streamer (NemotronStreamer, Sources/DictatorCore/Nemotron/NemotronStreamer.swift:16-163)
 *
 * The live chunk walk of one stream (drainChunks, NemotronStreamer.swift:109-154): the stream has consumed `idx`
 * of the `avail` mel rows it has so far; `last` says no more rows will come. Returns 1 when a chunk is ready:
 * rows [*start, *start + *valid_rows) (the first chunk 1+8R rows with no pre-encode cache, later chunks 9
 * cached rows + 8+8R new rows, run as soon as they exist; the final chunk shorter) followed by
 * *n_rows - *valid_rows zero rows that extend a final tail shorter than the minimum chunk (8 rows, 1 for a first
 * chunk) when end_padding != 0 (the reference's endPadding, :29-31; with end_padding 0 such a tail is dropped
 * as NeMo's batch-1 schedule and runBuffered, :70-91, do), *keep_all (the final chunk) and *next_idx. Returns 0
 * when the stream must wait for rows, -1 when it has ended. */
UD_API int ud_chunk_next(int lookahead, int idx, int avail, int last, int end_padding, int* start, int* n_rows,
                         int* valid_rows, int* keep_all, int* next_idx);

/* A streamer drives many streams of one engine: each step runs every stream with a ready chunk in one batched
 * encoder pass (ud_step_batch, with greedy RNN-T decoding when decode != 0) and appends the tokens to the
 * stream. A stream takes mel rows from a caller-owned host buffer [capacity_rows, mel_bins] that stays valid
 * until the stream is released (rows become available through ud_streamer_push), or audio through a mel
 * frontend of the same engine (ud_streamer_open_audio / ud_streamer_push_audio, NemotronStreamer.push(samples:)
 * and flush(), :95-107). A stream's engine slot is taken at open (UD_ERR_POOL_EXHAUSTED when the engine has none
 * free) and freed when its final chunk has run. End padding is on by default. Calls on one streamer are
 * serialised by the caller. */
typedef struct ud_streamer ud_streamer;
typedef int32_t ud_streamer_id;
UD_API ud_status ud_streamer_create(ud_engine* e, int lookahead, int decode, ud_streamer** out);
UD_API ud_status ud_streamer_destroy(ud_streamer* s);
UD_API ud_status ud_streamer_set_end_padding(ud_streamer* s, int on);
UD_API ud_status ud_streamer_open(ud_streamer* s, const float* mel, int capacity_rows, ud_streamer_id* out);
/* n_rows more rows are valid at the end of the stream's buffer; last != 0: the stream ends there. */
UD_API ud_status ud_streamer_push(ud_streamer* s, ud_streamer_id id, int n_rows, int last);
/* An audio stream: its mel comes from frontend `mel` (one frontend for all audio streams of a streamer). */
UD_API ud_status ud_streamer_open_audio(ud_streamer* s, ud_mel* mel, ud_streamer_id* out);
/* n_samples[i] more samples of stream ids[i] (one frontend call for all of them); last[i] != 0 ends the stream
 * (NemotronStreamer.flush). last may be NULL. */
UD_API ud_status ud_streamer_push_audio(ud_streamer* s, int n, const ud_streamer_id* ids, const float* const* samples,
                                        const int* n_samples, const int* last);
/* One batched step (at most max_batch streams, in order of id); *n_stepped streams advanced one chunk,
 * *n_finished of them ran their final chunk (or ended with nothing left to encode). */
UD_API ud_status ud_streamer_step(ud_streamer* s, int* n_stepped, int* n_finished);
/* Pipelined steps (a decoding streamer only; off by default): each ud_streamer_step issues its batch with
 * ud_step_batch_async from pinned staging buffers and takes in the results of the step before it, so the
 * host's chunk gathering and the copies overlap the device's work. A step's tokens, emission records and
 * finished streams appear one ud_streamer_step later (a step with no ready stream only completes the one in
 * flight). Token sequences are those of the synchronous mode. Turning it off completes the step in flight. */
UD_API ud_status ud_streamer_set_pipelined(ud_streamer* s, int on);
/* The ids of the streams that finished in the last ud_streamer_step (up to cap copied) and their count. */
UD_API ud_status ud_streamer_finished(ud_streamer* s, ud_streamer_id* out, int cap, int* n);
/* Tokens so far (up to cap copied), the total count, and whether the stream has finished. */
UD_API ud_status ud_streamer_tokens(ud_streamer* s, ud_streamer_id id, int32_t* out, int cap, int* n_tokens,
                                    int* finished);
/* Emission records (Emission, Sources/DictatorCore/Nemotron/Streaming.swift:6-15, filled as drainChunks does,
 * NemotronStreamer.swift:141): for each token so far, the input the stream had received when the step that
 * emitted it ran (audio samples for an audio stream; 160 x the mel rows pushed for a mel stream) and that step's
 * wall seconds (its batched encoder pass and decoding). Up to cap of each copied (any pointer may be NULL);
 * *n = the token count. */
UD_API ud_status ud_streamer_emissions(ud_streamer* s, ud_streamer_id id, int32_t* tokens, int64_t* samples_seen,
                                       double* compute_seconds, int cap, int* n);
/* Wall seconds of each step the stream took part in (NemotronStreamer.wallTimes, :24-25, 63); *n = count. */
UD_API ud_status ud_streamer_step_times(ud_streamer* s, ud_streamer_id id, double* out, int cap, int* n);
/* Forgets a stream (closing its engine slot if it has not finished); its id may be reused. */
UD_API ud_status ud_streamer_release(ud_streamer* s, ud_streamer_id id);

/* ---- SentencePiece detokenizer (SentencePieceDecoder, Sources/DictatorCore/Text/SentencePiece.swift:5-32)
 *
 * Host code, no GPU. The vocabulary is the tokenizer.vocab text: one "piece\tscore" line per id, empty lines
 * skipped. Decoding joins the pieces of the valid ids: "<0xHH>" pieces give the byte, <unk> <s> </s> <pad>
 * nothing, other pieces their UTF-8 with U+2581 turned into a space; ill-formed UTF-8 becomes U+FFFD and one
 * leading space is dropped. ud_detok_decode writes at most cap - 1 bytes plus a NUL and the full length to
 * *len_out (call with cap 0 to size the buffer). */
typedef struct ud_detok ud_detok;
UD_API ud_status ud_detok_create(const char* vocab_text, size_t len, ud_detok** out);
UD_API ud_status ud_detok_create_file(const char* path, ud_detok** out);
UD_API ud_status ud_detok_destroy(ud_detok* d);
UD_API int ud_detok_size(const ud_detok* d);
UD_API ud_status ud_detok_decode(const ud_detok* d, const int32_t* ids, int n, char* out, size_t cap,
                                 size_t* len_out);

/* Text of the last error on this thread ("" if none). Returns the full length. */
UD_API size_t ud_last_error(char* buf, size_t len);
UD_API const char* ud_status_string(ud_status s);

#ifdef __cplusplus
}
#endif

#endif /* UD_H */
