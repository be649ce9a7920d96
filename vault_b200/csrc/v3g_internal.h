// Host-side structures and cross-file entry points of the engine (not part of the public C ABI).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/vault_b200.h"
#include "v3g.cuh"
#include "v3g_gemm.cuh"
#include "v3g_gemv.cuh"

struct v3g_model {
    v3g::ModelDev host;              // host copy of the device descriptor
    v3g::ModelDev *dev = nullptr;    // device copy
    int device = 0;
    int n_sm = 148;
    uint8_t *weights = nullptr;      // one allocation holding every tile buffer and vector
    size_t weight_alloc = 0;
    // per-step algorithmic bytes (file payload bytes of every tensor streamed in a decode step)
    uint64_t step_bytes = 0, step_bytes_lm = 0, scorer_bytes = 0;
    uint32_t bos_id = 0, eos_id = 0, weight_format = 0, flags = 0;
    uint32_t file_seg_budget = 0;
    std::vector<std::pair<uint32_t, v3g::MatW *>> tensor_index;  // tensor id -> matrix (tests / sweeps)
    std::string last_error;
};

// chunked-prefill workspace inside the state arena: up to `cap` tokens (all sequences of a piece together)
struct PfBuf {
    int cap = 0;
    float *x = nullptr;      // [cap][d] residual stream of the piece's tokens
    float *qc = nullptr;     // [cap][H][D] queries rotated at their chunk position c
    float *qf = nullptr;     // [cap][H][D] queries rotated at W + c
    float *attn = nullptr;   // [cap][H D] attention outputs
    float *h = nullptr;      // [cap][F] SwiGLU activations
    __half *x16 = nullptr;   // [cap][ldx16] fp16 GEMM operand
    int ldx16 = 0;
    float *xscale = nullptr; // [cap] per-token operand scale
    float *feat = nullptr;   // [cap][feat_dim] segment-scorer features of every token
    float *hin = nullptr;    // [cap][feat_dim] habituated scorer inputs
    float *z = nullptr;      // [cap][2][seg_hidden] scorer fc1 outputs (raw, habituated)
    float4 *stat = nullptr;  // [cap] scorer LayerNorm statistics (means raw / habituated, inverse deviations)
    v3g::TcSplitWs sk;       // split-K partials and tickets of the tensor-core GEMM
};

struct v3g_state {
    const v3g_model *m = nullptr;
    v3g::StateDev host;
    v3g::StateDev *dev = nullptr;
    uint8_t *arena = nullptr;
    size_t arena_size = 0;
    int B = 1;
    int seg_cap = 0;                 // bank rows reserved per sequence
    int per_seq_memory = 0;          // batch > 1 with segment memory + auto-pin per sequence
    int auto_pin = 1;
    uint64_t pos = 0;                // host mirror of StepCtl::pos
    int seg_budget = 0;
    cudaStream_t cap_stream = nullptr;
    cudaGraphExec_t graphs[4] = {nullptr, nullptr, nullptr, nullptr};  // [boundary][with lm head]
    uint64_t graph_B_pos[4] = {0, 0, 0, 0};
    int use_graphs = 1;
    int use_pdl = 1;                 // programmatic dependent launch between the kernels of a step
    // persistent decode kernel (all layers + lm head in one cooperative launch)
    int use_mega = 0;
    void *mk_phases = nullptr;       // device MkPhase[mk_n]; the last entry is the lm head
    void *mk_lite = nullptr;         // device MkLite[mk_n] (chunk-stream table)
    void *mk_fn = nullptr;           // kernel instantiation for this model's head size and tile formats
    int mk_n = 0, mk_grid = 0, mk_slots = 0, mk_xr = 0;
    int mk_ph_off = 0, mk_lite_off = 0, mk_part_off = 0, mk_misc_off = 0, mk_nw_off = 0, mk_ring_off = 0,
        mk_bar_off = 0;
    size_t mk_smem = 0;
    PfBuf pf;
    int chunked_prefill = 1;         // v3g_prefill runs window-aligned pieces through the tensor-core GEMMs
    int use_tc_step = 0;             // batch > 8: decode steps run their projections on the tensor-core GEMM
    int act_single = 0;              // GEMV activations as one fp16 part (V3G_STATE_FP16_ACTIVATIONS)
    std::string last_error;
};

// records msg as this thread's v3g_last_error() and returns code
int v3g_fail(int code, const std::string &msg);
// validate a VLT3 buffer (no CRC pass) and return its VTOK tokenizer blob (v3g_api.cu)
int vlt3_token_blob(const uint8_t *buf, uint64_t size, const uint8_t **tok, uint64_t *tok_size);

namespace v3g {
int repack_matrix(MatW &w, const uint8_t *dev_src0, const uint8_t *dev_src1, int fmt, int src_rows, int cols,
                  int rowmap, int head_dim, uint8_t *dst, cudaStream_t st);
size_t matrix_tile_bytes(int fmt, int rows, int cols);
int dequant_matrix(const MatW &w, int head_dim, float *out, cudaStream_t st);

// one decode step for the whole batch (kernels only; the caller updates the host pos mirror)
cudaError_t launch_step(const v3g_model *m, v3g_state *s, bool boundary, bool want_lm, cudaStream_t st);
cudaError_t launch_prefix_refresh(const v3g_model *m, v3g_state *s, cudaStream_t st);
cudaError_t launch_state_reset(const v3g_model *m, v3g_state *s, cudaStream_t st);
cudaError_t init_kernel_attrs();
// persistent decode kernel set-up for a state (sets s->use_mega when the model / batch qualify)
cudaError_t build_mega(const v3g_model *m, v3g_state *s);
cudaError_t launch_mega(const v3g_model *m, v3g_state *s, bool want_lm, cudaStream_t st);
cudaError_t launch_attention(const v3g_model *m, v3g_state *s, int layer, bool pdl, cudaStream_t st);
cudaError_t launch_argmax_finish(const v3g_model *m, v3g_state *s, bool want_lm, bool pdl, cudaStream_t st);
cudaError_t launch_gemv_mapped(const v3g_model *m, const MatW &w, const float *x, int B, float *y, cudaStream_t st);
cudaError_t launch_gemv_store(const v3g_model *m, const MatW &w, const float *x, int B, float *y, cudaStream_t st);
// chunk-boundary kernels of a step at a window boundary (auto-pin of the boundary token, segment eviction, prefix
// re-rotation); the step's own kernels follow
cudaError_t launch_boundary(const v3g_model *m, v3g_state *s, cudaStream_t st);
// final RMSNorm + tied lm head of B rows (row b at x + b * x_ld) into the state's logits, and their argmax keys
cudaError_t launch_lm_head(const v3g_model *m, v3g_state *s, const float *x, int x_ld, cudaStream_t st);
cudaError_t launch_argmax_only(const v3g_model *m, v3g_state *s, cudaStream_t st);
// top-k + temperature draw per logit row (v3g_sample.cu); out, when not null, also receives row b's token at
// out[b * out_ld]
cudaError_t launch_sample_topk(const float *logits, uint32_t rows, uint32_t vocab, uint64_t ld, uint32_t k, float temp,
                               uint64_t *rng, int32_t *tokens, int32_t *out, int64_t out_ld, cudaStream_t st);
// governor masking / commit over rows of logits and stream states (v3g_sample.cu); no launch while n_rules == 0
cudaError_t launch_govern(const v3g_model *m, const v3g_gov_rules_t &rules, const v3g_gov_stream_t *streams,
                          float *logits, uint32_t rows, uint64_t ld, uint32_t top_k_guard, cudaStream_t st);
cudaError_t launch_gov_commit(const v3g_model *m, const v3g_gov_rules_t &rules, v3g_gov_stream_t *streams,
                              const int32_t *tokens, uint32_t rows, cudaStream_t st);
cudaError_t launch_step_begin(const v3g_model *m, v3g_state *s, bool boundary, cudaStream_t st);
cudaError_t launch_scorer(const v3g_model *m, v3g_state *s, cudaStream_t st);
// batched decode step (B > 8) with every projection on the tensor-core GEMM (v3g_prefill.cu)
cudaError_t launch_step_tc(const v3g_model *m, v3g_state *s, bool boundary, bool want_lm, cudaStream_t st);
bool step_tc_supported(const v3g_model *m, const v3g_state *s);
cudaError_t launch_step_attention(const v3g_model *m, v3g_state *s, int layer, cudaStream_t st);
cudaError_t tc_init_attrs();
// chunked prefill (v3g_prefill.cu)
bool piece_supported(const v3g_model *m, const v3g_state *s);
cudaError_t launch_piece(const v3g_model *m, v3g_state *s, const int32_t *dev_ids, int64_t ld, int64_t i0, int n,
                         int64_t p0, bool want_lm, cudaStream_t st);
}  // namespace v3g
