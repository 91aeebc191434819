// Launch interfaces of the libud kernels (host side). All kernels are sm_100a.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ud {

using bf16 = __nv_bfloat16;

enum Act : int { ACT_NONE = 0, ACT_RELU = 1, ACT_SILU = 2 };

// Launches a kernel of the step with programmatic stream serialization (the kernel calls pdl_wait before reading
// what earlier kernels wrote). Off when the environment sets UD_PDL=0.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, args...);
}

// C = out_scale * act(A . W^T + bias) + res_scale * R   (the contract of the reference's Step.gemm,
// Sources/DictatorEngine/Core/Kernels.swift:79-113, minus alpha which Nemotron never sets).
struct GemmEpilogue {
    const float* bias = nullptr;     // [N] or null
    int act = ACT_NONE;
    float out_scale = 1.f;
    const float* residual = nullptr; // fp32 [M, ldr] or null; may alias out (read before write, same thread)
    int ldr = 0;
    float res_scale = 1.f;
    void* out = nullptr;             // fp32 or bf16 [M, ldo]
    int ldo = 0;
    int out_bf16 = 0;
    // Graph-mode timer slot (2-CTA GEMM only, null when off; timer_start / timer_end in common.cuh).
    unsigned long long* prof = nullptr;
};

// ---- tcgen05 GEMM (bf16 x bf16 -> fp32 in TMEM), A [M, K] row-major (lda), W [N, K] row-major.
// Requirements: K % 64 == 0, N % 128 == 0, lda/ldw multiples of 8 elements, 16-byte aligned bases.
struct TmaMatrix {
    CUtensorMap map;
    const void* base = nullptr;
    int rows = 0, cols = 0, ld = 0, box_rows = 0;
};
bool make_tma_bf16(TmaMatrix& t, const void* base, int rows, int cols, int ld, int box_rows);
// Epilogue blocks: 32 rows x 128 bytes (32 fp32 or 64 bf16 columns), 128-byte swizzle, for TMA stores of GEMM
// outputs.
bool make_tma_epi(TmaMatrix& t, const void* base, int rows, int cols, int ld, bool bf16);
// K/V page pool [pages_total][page_frames][cols] bf16 as the 3-D tensor (column, frame, page): boxes of 64 columns x
// page_frames frames x 1 page, 128-byte swizzle. A load may start at a negative or past-the-end frame or page
// coordinate: those rows arrive as zeros.
bool make_tma_pages(TmaMatrix& t, const void* base, int pages_total, int page_frames, int cols);
int gemm_tc_pick_bn(int M, int N, int num_sms);
void gemm_tc(const TmaMatrix& A, const TmaMatrix& W, int M, int N, int K, int bn, const GemmEpilogue& epi,
             int* dev_err, int num_sms, cudaStream_t s);

// 2-CTA variant (cluster of 2, cta_group::2), 256 x bn tiles per CTA pair; bn must be 256 and W's tensor map
// must have 128-row boxes (each CTA loads half of the W tile). M >= 256 recommended.
// out_map (may be null): the epilogue tensor map of epi.out (make_tma_epi); bf16 outputs without a residual are
// then stored through TMA when every tile is 256 wide.
void gemm_tc2(const TmaMatrix& A, const TmaMatrix& W_half, int M, int N, int K, int bn, const GemmEpilogue& epi,
              int* dev_err, int num_sms, const TmaMatrix* out_map, cudaStream_t s);

// ---- SIMT GEMM for few rows (M small) and for the fp32 engine. TA/TW in {float, bf16}.
template <typename TA, typename TW>
void gemm_simt(const TA* A, int lda, const TW* W, int M, int N, int K, const GemmEpilogue& epi, cudaStream_t s);

// ---- LayerNorm over rows of width D (eps 1e-5). x fp32 [M, D] -> y (TO) [M, D].
template <typename TO>
void layer_norm(const float* x, const float* g, const float* b, TO* y, int M, int D, cudaStream_t s,
                unsigned long long* timer = nullptr);
// x <- LN1(x) (fp32, in place), y <- LN2(x) in TO: a layer's norm_out fused with the next layer's norm_ff1.
template <typename TO>
void layer_norm2(float* x, const float* g1, const float* b1, const float* g2, const float* b2, TO* y, int M, int D,
                 cudaStream_t s, unsigned long long* timer = nullptr);

// ---- Per-stream step metadata, uploaded once per batched step.
constexpr int kPageSlots = 8;     // page-table slots per stream (ring of pages)
struct BatchEntry {
    int slot;        // stream slot (index into per-slot arrays: conv cache, decoder state)
    int row_off;     // first row of this stream's frames in the packed [M, D] activations
    int T;           // frames this step
    int valid_t;     // valid frames (<= T)
    int cache_len;   // cached frames before this step (<= L)
    int head;        // absolute frame index of the first new frame (= frames appended so far)
    int drop;        // subsampled frames dropped from the front (0 first step, 2 later)
    int valid_mel;   // valid mel rows
    int n_rows;      // mel rows
    int keep;        // frames kept for the joint / decoder
    int tok_off;     // offset of this stream's token output
    int pad;
    int pages[kPageSlots];  // physical page per ring slot (-1 = unmapped)
};

struct CacheGeom {
    void* kpool;      // [n_layers][n_pages][page_frames][D] (engine dtype)
    void* vpool;
    void* conv;       // [n_layers][max_streams][conv_ring][D]
    int n_layers, n_pages, page_frames, D, L, conv_ring, max_streams;
};

// ---- Rel-pos attention over [cached window ; new chunk] with the fused append of the new K/V rows.
template <typename T>
void relpos_attention(const T* qkv, int ld_qkv, const T* ptab, int tmax, const float* bias_u, const float* bias_v,
                      const BatchEntry* meta, int n, int tmax_batch, const CacheGeom& cg, int layer, T* out,
                      int ldo, int n_heads, int* dev_err, cudaStream_t s);

// ---- Conv module core: GLU -> pad mask -> [conv cache ; new] -> depthwise k -> LN -> SiLU, cache update.
template <typename T>
void conv_module(const T* pw, int ld_pw, const float* dw, const float* ln_g, const float* ln_b,
                 const BatchEntry* meta, int n, int tmax_batch, const CacheGeom& cg, int layer, int K, T* out,
                 int ldo, int* dev_err, cudaStream_t s, unsigned long long* timer = nullptr);

// ---- Subsampling (causal dw-striding x8, channel-last activations [b][t][f][c]).
// conv0 + ReLU fused with the stage-1 depthwise conv: mel [n][rows_stride][mel_bins] -> out [n][T2][F2][C].
template <typename T>
void sub_conv01(const float* mel, int rows_stride, int mel_bins, const BatchEntry* meta, int n, int Tin, const float* w0,
                const float* b0, int T1, int F1, const float* w1, const float* b1, T* out, int T2, int F2, int C,
                int num_sms, cudaStream_t s);
// Stage-2 depthwise conv: in [n][Tin][Fin][C] -> out [n][Tout][Fout][C].
template <typename T>
void sub_dwconv2(const T* in, int Tin, int Fin, const BatchEntry* meta, int n, const float* w, const float* b, T* out,
                 int Tout, int Fout, int C, cudaStream_t s);
template <typename T>
void sub_select(const float* sub_out, int T3, const float* out_bias, const BatchEntry* meta, int n, float* x,
                int D, cudaStream_t s);

// ---- Cache ops (microbenchmark / tests). rows are engine dtype.
template <typename T>
void cache_append(const T* kv_rows, const T* conv_rows, int k, const BatchEntry* meta, int n, const CacheGeom& cg,
                  int* dev_err, cudaStream_t s);
template <typename T>
void cache_gather(T* kv_out, T* conv_out, const BatchEntry* meta, int n, const CacheGeom& cg, int* dev_err,
                  cudaStream_t s);
template <typename T>
void conv_slot_zero(const int* slots, int n, const CacheGeom& cg, cudaStream_t s);

// ---- RNN-T greedy (fused prediction LSTM + joint + argmax loop), one CTA per stream.
struct RnntWeights {
    const float* embed;    // [V, Hp]
    const float* w_ih[4];  // [4Hp, Hp]
    const float* w_hh[4];  // [4Hp, Hp]
    const float* bias[4];  // [4Hp] = b_ih + b_hh
    const float* pred_w;   // [J, Hp]
    const float* pred_b;   // [J]
    const float* out_w;    // [V, J]
    const float* out_b;    // [V]
    int layers, Hp, J, V, max_symbols;
};
struct RnntState {         // per slot
    float* h;              // [slots][layers][Hp]
    float* c;
    float* pend_g;         // [slots][J]
    float* pend_h;         // [slots][layers][Hp]
    float* pend_c;
    int* last_tok;         // [slots]
    int* pend_valid;       // [slots]
};
// Scratch of the lock-step decoder (all streams of a batch advance frame by frame together, every SM holding a
// slice of the LSTM, prediction and joint rows in shared memory; grid barriers between the stages).
struct RnntScratch {
    unsigned long long* barrier = nullptr;  // grid-barrier arrival counter, zeroed before each launch
    int* done_frame = nullptr;              // [max_n] frames a stream has finished in this launch
    int* emitted = nullptr;                 // [max_n] symbols emitted in the current frame
    float* part_val = nullptr;              // [max_n * max_grid] per-CTA joint maxima
    int* part_idx = nullptr;                // [max_n * max_grid] their vocabulary ids
    int max_n = 0, max_grid = 0;
    int lockstep_max_n = 64;   // larger batches decode faster with one CTA per stream (grid full, weights in L2)
    int tc_min_n = 20;         // batches of at least this many streams decode on the tensor cores (below it the fp32
                               // lock-step kernel is faster: the per-iteration cost of the tensor-core one is fixed)
    struct RnntTc* tc = nullptr;   // operands of the tensor-core decoder (null: off)
};
// Operands of the tensor-core decoder (rnnt_tc.cu). Each fp32 value x is carried as two fp16 values,
// hi = fp16(x) and lo = fp16((x - hi) * 2^11), so x = hi + lo * 2^-11 to within 2^-22 |x|.
struct RnntTc {
    // The weights, split at load: LSTM layer l as [4Hp][2Hp], rows unit-major (row 4u + q is gate q of unit u),
    // K = [w_ih row ; w_hh row]; joint.pred [J][Hp]; the joint output [V][J].
    uint16_t* wl_hi[4] = {};
    uint16_t* wl_lo[4] = {};
    uint16_t *wp_hi = nullptr, *wp_lo = nullptr, *wo_hi = nullptr, *wo_lo = nullptr;
    bool weights_ok = false;   // split, with every weight and embedding value inside the fp16 range
    // Per-stream operand rows in batch order (n_pad rows, zero at allocation): the LSTM inputs [x_l ; h_l], the
    // prediction input h_top and the joint input relu(f_t + g).
    uint16_t* xl_hi[4] = {};
    uint16_t* xl_lo[4] = {};
    uint16_t *xp_hi = nullptr, *xp_lo = nullptr, *xj_hi = nullptr, *xj_lo = nullptr;
    int n_pad = 0;
    TmaMatrix m_xl_hi[4], m_xl_lo[4], m_xp_hi, m_xp_lo, m_xj_hi, m_xj_lo;   // boxes of 128 rows
    bool maps_ok = false;
    TmaMatrix m_wl_hi[4], m_wl_lo[4], m_wp_hi, m_wp_lo, m_wo_hi, m_wo_lo;   // boxes of one slice width
    int bn_lstm = 0, bn_pred = 0, bn_joint = 0;                             // slice widths of those maps
};
// Host splits of weights into the decoder's pairs (hi, lo of `count` values; the LSTM as unit-major [4Hp][2Hp]
// rows); false if a value is beyond the fp16 range.
bool rnnt_tc_split(const float* w, size_t count, uint16_t* hi, uint16_t* lo);
bool rnnt_tc_split_lstm(const float* w_ih, const float* w_hh, int Hp, uint16_t* hi, uint16_t* lo);
// The tensor maps of the operand rows (after the row buffers are allocated).
bool rnnt_tc_build_row_maps(RnntTc& tc, int layers, int Hp, int J);
// Greedy decoding of n streams. With scr: batches of at least scr->tc_min_n streams run the tensor-core lock-step
// decoder (rnnt_tc.cu) when its shape limits hold; else, with n <= scr->lockstep_max_n and weights whose slices fit
// in shared memory, the fp32 lock-step kernel on min(num_sms, scr->max_grid) CTAs; otherwise one CTA per stream.
void rnnt_greedy(const RnntWeights& w, const RnntState& st, const float* proj, int ld_proj, const BatchEntry* meta,
                 int n, int32_t* tokens, int tok_stride, int* n_tokens, const RnntScratch* scr, int num_sms,
                 int* dev_err, cudaStream_t s);
// The tensor-core lock-step decoder; returns false, launching nothing, outside its limits (operands split and mapped,
// Hp and J multiples of 64, at most 4 LSTM layers, n <= scr.max_n and the row buffers, V <= 16 x grid).
bool rnnt_greedy_tc(const RnntWeights& w, const RnntState& st, const float* proj, int ld_proj, const BatchEntry* meta,
                    int n, int32_t* tokens, int tok_stride, int* n_tokens, const RnntScratch& scr, int num_sms,
                    int* dev_err, cudaStream_t s);
void rnnt_reset(const RnntState& st, const int* slots, int n, const RnntWeights& w, cudaStream_t s);

void pack_frames(const float* frames, int rows_stride, const BatchEntry* meta, int n, int tmax, float* x, int D,
                 cudaStream_t s);
void scatter_rows(const float* src, const BatchEntry* meta, int n, float* dst, int tmax, int W, cudaStream_t s);
size_t relpos_attention_smem_bytes(int tmax_batch, int L, int elem_bytes);
// The bf16 attention as a persistent TMA-fed kernel (attention.cu): qkv [rows, 3 D] (box 64 x 16), the K and V page
// pools (make_tma_pages, 16-frame pages) and this layer's position table (box 64 x 128, from row ptab_row0 =
// tmax - 16). Returns false, launching nothing, when the shapes are outside its limits (chunks of more than 16
// frames, pages of other than 16 frames, L + 15 beyond the 128 staged position rows).
bool relpos_attention_tma(const TmaMatrix& qkv, const TmaMatrix& kpool, const TmaMatrix& vpool, const TmaMatrix& ptab,
                          int ptab_row0, const float* bias_u, const float* bias_v, const BatchEntry* meta, int n,
                          int tmax_batch, const CacheGeom& cg, int layer, bf16* out, int ldo, int n_heads, int num_sms,
                          int* dev_err, cudaStream_t s, unsigned long long* timer = nullptr);
size_t rnnt_smem_bytes(const RnntWeights& w);

// ---- misc
void fill_f32(float* p, float v, size_t n, cudaStream_t s);
void f32_to_bf16(const float* in, bf16* out, size_t n, cudaStream_t s);
void test_wait_timeout(int* dev_err, uint64_t limit_ns, cudaStream_t s);

}  // namespace ud
