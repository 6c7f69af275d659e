// model.cu -- the model_* C ABI (include/model.h, include/tie_b200.h) on one B200.
//
// Host orchestration only: argument checks in the reference's order, the
// load-time upload of the weights to device memory, scratch management, and the
// launch sequence of the forward pass. Every arithmetic step of the token loop
// is a kernel (k_*.cu).
//
// Reference correspondence (src/model.c):
//   model_load            331-467   config + inventory + weight file, cross-checked
//   model_reserve         566-589   device scratch instead of host scratch
//   forward (prefill)     647-763   launch sequence in run_prefill()
//   cached decode         794-868   launch sequence in run_decode()
//   model_prefill         765-782, model_decode_step_cached 870-896,
//   model_decode_step     898-918, model_argmax 920-925
#include "../../include/model.h"
#include "../../include/safetensors.h"
#include "../../include/tie_b200.h"
#include "internal.h"
#include "json_doc.h"
#include "tc_gemm.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <new>
#include <string>
#include <vector>

using namespace tie;

namespace {

// ------------------------------------------------------------- artifacts --
// config.json and the tensor inventory are parsed whole into JSON trees
// (json_doc.h) and read by field; the inventory's "tensors" array is indexed
// by name once per load.

// A tensor as the inventory describes it.
struct TensorInfo {
    std::string dtype, orientation;
    std::vector<long long> shape;
    unsigned long long file_offset = 0, nbytes = 0;
};

// Integer-valued fields are read as numbers and truncated toward zero, as a
// C (int) conversion of the parsed value would.
bool field_int(const json::Value& obj, const char* key, int* out) {
    const json::Value* v = obj.get(key);
    if (!v || !v->is_number()) return false;
    *out = (int)v->num;
    return true;
}

bool field_u64(const json::Value& obj, const char* key, unsigned long long* out) {
    const json::Value* v = obj.get(key);
    if (!v || !v->is_number() || v->num < 0) return false;
    *out = (unsigned long long)v->num;
    return true;
}

bool field_str(const json::Value& obj, const char* key, std::string* out) {
    const json::Value* v = obj.get(key);
    if (!v || !v->is_string()) return false;
    *out = v->str;
    return true;
}

class Inventory {
  public:
    // false when the text is not JSON or has no "tensors" array of named records
    bool parse(const std::string& text) {
        if (!json::parse(text.data(), text.size(), &doc_) || doc_.kind != json::Kind::Object) return false;
        const json::Value* list = doc_.get("tensors");
        if (!list || list->kind != json::Kind::Array) return false;
        for (const json::Value& rec : list->items) {
            const json::Value* name = rec.get("name");
            if (name && name->is_string()) by_name_.emplace(name->str, &rec);
        }
        return true;
    }
    // The record of `name`, or false when it is absent or incomplete.
    bool find(const std::string& name, TensorInfo* t) const {
        auto it = by_name_.find(name);
        if (it == by_name_.end()) return false;
        const json::Value& rec = *it->second;
        *t = TensorInfo();
        if (!field_str(rec, "dtype", &t->dtype) || !field_str(rec, "orientation", &t->orientation) ||
            !field_u64(rec, "file_offset", &t->file_offset) || !field_u64(rec, "nbytes", &t->nbytes))
            return false;
        const json::Value* sh = rec.get("shape");
        if (!sh || sh->kind != json::Kind::Array || sh->items.size() > 8) return false;
        for (const json::Value& d : sh->items) {
            if (!d.is_number()) return false;
            t->shape.push_back((long long)d.num);
        }
        return true;
    }
    // The config values the inventory was produced against, or nullptr.
    const json::Value* config_values() const {
        const json::Value* cv = doc_.get("config_values_used");
        return cv && cv->kind == json::Kind::Object ? cv : nullptr;
    }

  private:
    json::Value doc_;
    std::map<std::string, const json::Value*> by_name_;
};

struct Layer {
    float *ln1_w, *ln1_b, *qkv_w, *qkv_b, *proj_w, *proj_b;
    float *ln2_w, *ln2_b, *fc_w, *fc_b, *mlp_w, *mlp_b;
    // tf32 splits (hi + lo == the fp32 weight) of the four matrices, for the
    // tensor-core matmul
    float *qkv_hi, *qkv_lo, *proj_hi, *proj_lo, *fc_hi, *fc_lo, *mlp_hi, *mlp_lo;
};

// A reduced-format matrix as the small-batch decode streams it.
struct QMat {
    int wt = WF_F32;              // WF_BF16 or WF_INT8 (WF_F32: use the fp32 weights)
    const void* q = nullptr;      // [out][in] bf16 or int8
    const float* s = nullptr;     // [out] int8 scales
};

// One reduced weight format (k_quant.cu): the compact copies of the five
// matrix kinds (qkv, proj, fc, mlp per layer; the tied wte) and the fp32
// weights they stand for, with their tf32 splits, which every other path uses
// while the format is selected. Vectors (LayerNorm, biases) and wpe stay fp32.
struct WeightSet {
    void* block = nullptr;
    size_t bytes = 0;
    std::vector<Layer> layers;    // fp32 view: the dequantised matrices
    float *wte = nullptr, *wte_hi = nullptr, *wte_lo = nullptr;
    std::vector<QMat> q;          // per layer: qkv, proj, fc, mlp; then wte
};

// A matmul operand: its fp32 values and/or its tf32 split.
struct Mat {
    const float* f;
    const float* hi;
    const float* lo;
};

// Decode batches of at most this many rows take the streaming GEMV; larger
// ones the tensor-core matmuls. Measured on B200 (GPT-2 small, each matmul
// alone): at 8 rows the two paths are level (QKV 10.1 vs 10.6 us, FC 9.7 vs
// 13.1, MLP 16.9 vs 13.3, head 87 vs 101), at 12-16 rows the GEMV is behind
// (QKV 14.9, FC 14.6, MLP 22.2, head 152 us at 16 rows), and a whole greedy
// step of 16 sequences took 1.21 ms on the GEMVs against 0.93 ms for 17 on
// the tensor cores.
constexpr int kGemvRows = 8;

// The tied head of decode steps of 9..kHeadTileRows rows takes tc_head_kernel:
// one MMA covers every row of the step, the vocabulary rows being the 128-row
// operand. (The layer matmuls keep the split-K kernel: with only 6-24 output
// tiles of 128 they need a cross-CTA reduction either way, and measured on
// B200 at 256 rows the transposed tile's reduction cost more than it saved.)
constexpr int kHeadTileRows = 256;

// CTAs a stream-kernel trace reserves per kernel (at most one per SM)
constexpr int kTraceCtas = 256;

// One instantiated decode graph per (batch size, cache, advance, output) key,
// with the number of kernels one replay runs.
struct GraphKey {
    int B;
    const kv_cache* cache;
    bool advance;
    const int32_t* out;
    int ld_out;
    bool operator<(const GraphKey& o) const {
        if (B != o.B) return B < o.B;
        if (cache != o.cache) return cache < o.cache;
        if (advance != o.advance) return advance < o.advance;
        if (out != o.out) return out < o.out;
        return ld_out < o.ld_out;
    }
};
struct GraphEntry {
    cudaGraphExec_t exec;
    uint64_t kernels;
};

}  // namespace

struct model {
    model_config cfg{};
    model_cproj_reading cproj = MODEL_CPROJ_AS_STORED;
    model_decode_path path = MODEL_PATH_NOCACHE;
    kv_cache* kv = nullptr;
    const gemm_impl* gemm_choice = &gemm_impl_sm100a;
    int device = 0;
    cudaStream_t st = nullptr;

    float* d_weights = nullptr;
    size_t weight_bytes = 0;
    float* d_split = nullptr;  // tf32 splits of every matrix
    size_t split_bytes = 0;
    float *wte = nullptr, *wpe = nullptr, *lnf_w = nullptr, *lnf_b = nullptr;
    float *wte_hi = nullptr, *wte_lo = nullptr;
    std::vector<Layer> layers;        // the selected weight format's fp32 view
    std::vector<model_tensor_record> records;
    // the weights as loaded, and the reduced formats built on request
    int wfmt = WF_F32;
    std::vector<Layer> base_layers;
    float *base_wte = nullptr, *base_wte_hi = nullptr, *base_wte_lo = nullptr;
    WeightSet sets[3];

    // activation scratch: `rows` rows
    size_t rows = 0;
    float *x = nullptr, *xb = nullptr, *qkv = nullptr, *attn = nullptr, *ff = nullptr;
    float *xb_hi = nullptr, *xb_lo = nullptr, *attn_hi = nullptr, *attn_lo = nullptr;
    float *ff_hi = nullptr, *ff_lo = nullptr;
    int* d_err = nullptr;        // set by a kernel whose bounded wait expired
    size_t logit_rows = 0;
    float* logits = nullptr;
    size_t ids_cap = 0;
    int32_t* d_ids = nullptr;

    // decode state (batch slots)
    size_t slots = 0;
    int32_t *d_tokens = nullptr, *d_lens = nullptr, *d_next = nullptr, *d_step = nullptr;
    size_t out_cap = 0;
    int32_t* d_out = nullptr;
    size_t part_floats = 0;
    float* d_part = nullptr;
    size_t cnt_cap = 0;
    int* d_attn_cnt = nullptr;  // per (sequence, head) arrival counters of the decode attention
    size_t am_parts = 0;
    float* d_am_val = nullptr;
    int* d_am_idx = nullptr;

    // pinned staging for small host<->device transfers
    int32_t* h_small = nullptr;
    size_t h_small_cap = 0;

    bool stats_on = false;
    AttnStats* d_stats = nullptr;
    double rs_min = 0.0, rs_max = 0.0;
    size_t rs_rows = 0;

    kv_cache* pool = nullptr;
    std::map<GraphKey, GraphEntry> graphs;

    // the persistent decode step (k_step.cu)
    int step_kind = TIE_STEP_CHAINED;
    StepLayer* d_step_layers = nullptr;
    unsigned* d_sync = nullptr;      // the step kernel's stage counters
    int step_state[5] = {0, 0, 0, 0, 0};  // per batch size: 0 unknown, 1 runs, -1 does not
    int step_slots[5] = {0, 0, 0, 0, 0};
    int step_grid = 0;
    uint64_t launches = 0;
    // failure drill: the next decode step's first matmul waits on a barrier
    // nothing completes, for at most drill_ns (model_debug_wait_drill)
    unsigned long long drill_ns = 0;
    // stream-kernel trace of one step (model_stream_trace): per stream kernel
    // in launch order, [grid][kStreamTraceEvents] stamps; NULL otherwise
    unsigned long long* stream_trace = nullptr;
    int stream_traced = 0;
};

namespace {

// The last CUDA error a model call hit on this thread (tie_last_device_error),
// and, with TIE_DEBUG set in the environment, one line per failure on stderr.
thread_local char g_dev_err[256] = "";

void note_cuda(cudaError_t e, const char* what, int line) {
    std::snprintf(g_dev_err, sizeof g_dev_err, "%s (%s) at model.cu:%d: %s", cudaGetErrorName(e),
                  cudaGetErrorString(e), line, what);
    static const bool verbose = std::getenv("TIE_DEBUG") != nullptr;
    if (verbose) std::fprintf(stderr, "tie_b200: %s\n", g_dev_err);
}

#define CU(expr)                                                   \
    do {                                                           \
        cudaError_t e_ = (expr);                                   \
        if (e_ != cudaSuccess) { note_cuda(e_, #expr, __LINE__); cudaGetLastError(); return MODEL_ERR_DEVICE; } \
    } while (0)

#define LAUNCH(expr)                                               \
    do {                                                           \
        cudaError_t e_ = (expr);                                   \
        ++m->launches;                                             \
        if (e_ != cudaSuccess) { note_cuda(e_, #expr, __LINE__); cudaGetLastError(); return MODEL_ERR_DEVICE; } \
    } while (0)

void drop_graphs(model* m) {
    for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second.exec);
    m->graphs.clear();
}

template <typename T>
model_status grow(T** p, size_t* cap, size_t need) {
    if (need <= *cap) return MODEL_OK;
    T* fresh = nullptr;
    if (cudaMalloc(&fresh, need * sizeof(T)) != cudaSuccess) { cudaGetLastError(); return MODEL_ERR_NOMEM; }
    cudaFree(*p);
    *p = fresh;
    *cap = need;
    return MODEL_OK;
}

model_status ensure_rows(model* m, size_t rows) {
    if (!m->d_err) {
        CU(cudaMalloc(&m->d_err, sizeof(int)));
        CU(cudaMemset(m->d_err, 0, sizeof(int)));
    }
    if (rows <= m->rows) return MODEL_OK;
    drop_graphs(m);
    const size_t E = (size_t)m->cfg.n_embd;
    // per row: x, xb, qkv (3E), attn, ff (4E), xb hi/lo, attn hi/lo, ff hi/lo (8E)
    const size_t per_row = E * (1 + 1 + 3 + 1 + 4 + 2 + 2 + 8);
    float* block = nullptr;
    if (cudaMalloc(&block, rows * per_row * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        return MODEL_ERR_NOMEM;
    }
    cudaFree(m->x);
    float* c = block;
    auto take = [&](size_t w) { float* p = c; c += rows * w; return p; };
    m->x = take(E); m->xb = take(E); m->qkv = take(3 * E); m->attn = take(E); m->ff = take(4 * E);
    m->xb_hi = take(E); m->xb_lo = take(E); m->attn_hi = take(E); m->attn_lo = take(E);
    m->ff_hi = take(4 * E); m->ff_lo = take(4 * E);
    m->rows = rows;
    return grow(&m->d_ids, &m->ids_cap, rows);
}

model_status ensure_logits(model* m, size_t rows) {
    if (rows <= m->logit_rows) return MODEL_OK;
    drop_graphs(m);
    size_t cap = m->logit_rows * (size_t)m->cfg.vocab_size;
    model_status rc = grow(&m->logits, &cap, rows * (size_t)m->cfg.vocab_size);
    if (rc == MODEL_OK) m->logit_rows = rows;
    return rc;
}

model_status ensure_pinned(model* m, size_t n_ints) {
    if (n_ints <= m->h_small_cap) return MODEL_OK;
    int32_t* p = nullptr;
    if (cudaMallocHost(&p, n_ints * sizeof(int32_t)) != cudaSuccess) { cudaGetLastError(); return MODEL_ERR_NOMEM; }
    cudaFreeHost(m->h_small);
    m->h_small = p;
    m->h_small_cap = n_ints;
    return MODEL_OK;
}

// Decode-state buffers for B sequences with a cache of `capacity` positions.
model_status ensure_slots(model* m, size_t B, int capacity) {
    model_status rc = ensure_rows(m, B);
    if (rc != MODEL_OK) return rc;
    if (B > m->slots) {
        drop_graphs(m);
        size_t c1 = m->slots, c2 = m->slots, c3 = m->slots;
        if ((rc = grow(&m->d_tokens, &c1, B)) != MODEL_OK) return rc;
        if ((rc = grow(&m->d_lens, &c2, B)) != MODEL_OK) return rc;
        if ((rc = grow(&m->d_next, &c3, B)) != MODEL_OK) return rc;
        m->slots = B;
    }
    if (!m->d_step) CU(cudaMalloc(&m->d_step, sizeof(int32_t)));
    if (!m->d_stats) CU(cudaMalloc(&m->d_stats, sizeof(AttnStats)));
    const size_t splits = (size_t)attn_decode_max_splits(capacity);
    const size_t need = B * (size_t)m->cfg.n_head * splits * (64 + 2 + 64);
    if (need > m->part_floats) {
        drop_graphs(m);
        if ((rc = grow(&m->d_part, &m->part_floats, need)) != MODEL_OK) return rc;
    }
    const size_t cnt = B * (size_t)m->cfg.n_head;
    if (cnt > m->cnt_cap) {
        drop_graphs(m);
        if ((rc = grow(&m->d_attn_cnt, &m->cnt_cap, cnt)) != MODEL_OK) return rc;
        CU(cudaMemset(m->d_attn_cnt, 0, cnt * sizeof(int)));
    }
    int sms = 0;
    CU(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, m->device));
    const size_t parts = (size_t)std::max({gemv_argmax_blocks(m->cfg.vocab_size),
                                           dec_head_blocks_max(m->cfg.vocab_size, m->cfg.n_embd), sms}) * B;
    if (parts > m->am_parts) {
        drop_graphs(m);
        size_t c1 = m->am_parts, c2 = m->am_parts;
        if ((rc = grow(&m->d_am_val, &c1, parts)) != MODEL_OK) return rc;
        if ((rc = grow(&m->d_am_idx, &c2, parts)) != MODEL_OK) return rc;
        m->am_parts = parts;
    }
    if ((rc = ensure_logits(m, B)) != MODEL_OK) return rc;
    return ensure_pinned(m, 2 * B + 16);
}

// Y (epilogue) = X . W^T over `rows` rows. Decode batches of at most kGemvRows
// rows take the streaming GEMV on fp32 operands; everything else takes the
// tensor-core matmul on tf32 splits (split over K, by N and K only, for
// decode-sized calls). Outputs: y (fp32) and/or y_hi/y_lo (its split).
model_status matmul(model* m, bool decode, int rows, Mat x, int ldx, Mat w, int N, int K,
                    const float* bias, int epi, float* y, float* y_hi, float* y_lo, int ldy) {
    cudaStream_t st = m->st;
    if (decode && rows <= kGemvRows) {
        LAUNCH(launch_gemv(x.f, ldx, w.f, K, bias, y, ldy, rows, N, K, epi, st));
        return MODEL_OK;
    }
    TcOperands op{x.hi, x.lo, ldx, w.hi, w.lo, K};
    TcArgs a{};
    a.M = rows; a.N = N; a.K = K; a.bias = bias;
    a.C = y; a.C_hi = y_hi; a.C_lo = y_lo; a.ldc = ldy;
    a.err = m->d_err;
    const int out = y_hi ? (y ? TC_OUT_F32_HILO : TC_OUT_HILO) : TC_OUT_F32;
    if (decode && epi == EPI_STORE && out == TC_OUT_F32 && rows <= kHeadTileRows) {
        // the tied head of a decode step: the vocabulary as the MMA's 128-row
        // operand, read as fp32 and split in shared memory
        op.b_f32 = w.f;
        LAUNCH(launch_tc_head(op, a, st));
        return MODEL_OK;
    }
    const int splits = decode ? tc_splits_for(N, K) : 1;
    LAUNCH(launch_tc_gemm(op, a, epi, out, splits, st));
    return MODEL_OK;
}

// ------------------------------------------------------------- stats --
model_status stats_begin(model* m) {
    if (!m->stats_on) return MODEL_OK;
    if (!m->d_stats) CU(cudaMalloc(&m->d_stats, sizeof(AttnStats)));
    AttnStats init{~0ull, 0ull, 0ull};
    CU(cudaMemcpyAsync(m->d_stats, &init, sizeof init, cudaMemcpyHostToDevice, m->st));
    CU(cudaStreamSynchronize(m->st));
    return MODEL_OK;
}

model_status stats_end(model* m) {
    if (!m->stats_on) return MODEL_OK;
    AttnStats s;
    CU(cudaMemcpy(&s, m->d_stats, sizeof s, cudaMemcpyDeviceToHost));
    if (s.rows) {
        double lo, hi;
        std::memcpy(&lo, &s.min_bits, 8);
        std::memcpy(&hi, &s.max_bits, 8);
        if (m->rs_rows == 0) { m->rs_min = lo; m->rs_max = hi; }
        else {
            if (lo < m->rs_min) m->rs_min = lo;
            if (hi > m->rs_max) m->rs_max = hi;
        }
        m->rs_rows += (size_t)s.rows;
    }
    return MODEL_OK;
}

// --------------------------------------------------------- forward passes --
// Prefill of n_seq sequences of T tokens whose ids are in m->d_ids; leaves
// LN_f(x) in m->xb. Keys and values go to `cache` when it is non-NULL
// (sequences first_seq..).                                   model.c:647-763
model_status run_prefill(model* m, int n_seq, int T, kv_cache* cache, int first_seq) {
    const int E = m->cfg.n_embd, H = m->cfg.n_head, R = n_seq * T;
    const float eps = m->cfg.layer_norm_epsilon;
    cudaStream_t st = m->st;
    AttnStats* stats = m->stats_on ? m->d_stats : nullptr;
    const Mat xb{nullptr, m->xb_hi, m->xb_lo}, attn{nullptr, m->attn_hi, m->attn_lo};
    const Mat ff{nullptr, m->ff_hi, m->ff_lo};
    model_status rc;
    LAUNCH(launch_embed_prefill(m->d_ids, R, T, m->wte, m->wpe, m->x, E, m->cfg.vocab_size, st));
    for (int l = 0; l < m->cfg.n_layer; ++l) {
        const Layer& w = m->layers[l];
        LAUNCH(launch_layernorm(m->x, w.ln1_w, w.ln1_b, nullptr, R, E, eps, st, m->xb_hi, m->xb_lo));
        if ((rc = matmul(m, false, R, xb, E, Mat{w.qkv_w, w.qkv_hi, w.qkv_lo}, 3 * E, E, w.qkv_b, EPI_BIAS,
                         m->qkv, nullptr, nullptr, 3 * E)) != MODEL_OK)
            return rc;
        if (cache) LAUNCH(launch_kv_store_prefill(m->qkv, n_seq, T, layer_view(cache, l), first_seq, st));
        LAUNCH(launch_attn_prefill(m->qkv, n_seq, T, H, nullptr, stats, st, m->attn_hi, m->attn_lo, m->d_err));
        if ((rc = matmul(m, false, R, attn, E, Mat{w.proj_w, w.proj_hi, w.proj_lo}, E, E, w.proj_b,
                         EPI_BIAS_RESID, m->x, nullptr, nullptr, E)) != MODEL_OK)
            return rc;
        LAUNCH(launch_layernorm(m->x, w.ln2_w, w.ln2_b, nullptr, R, E, eps, st, m->xb_hi, m->xb_lo));
        if ((rc = matmul(m, false, R, xb, E, Mat{w.fc_w, w.fc_hi, w.fc_lo}, 4 * E, E, w.fc_b, EPI_BIAS_GELU,
                         nullptr, m->ff_hi, m->ff_lo, 4 * E)) != MODEL_OK)
            return rc;
        if ((rc = matmul(m, false, R, ff, 4 * E, Mat{w.mlp_w, w.mlp_hi, w.mlp_lo}, E, 4 * E, w.mlp_b,
                         EPI_BIAS_RESID, m->x, nullptr, nullptr, E)) != MODEL_OK)
            return rc;
    }
    LAUNCH(launch_layernorm(m->x, m->lnf_w, m->lnf_b, nullptr, R, E, eps, st, m->xb_hi, m->xb_lo));
    return MODEL_OK;
}

// The tied head over `rows` rows of LN_f(x) starting at row `first` with row
// stride `stride` rows: logits [rows, V] into m->logits.
model_status prefill_head(model* m, int rows, size_t first, int stride) {
    const int E = m->cfg.n_embd, V = m->cfg.vocab_size;
    const size_t off = first * (size_t)E;
    return matmul(m, false, rows, Mat{nullptr, m->xb_hi + off, m->xb_lo + off}, stride * E,
                  Mat{m->wte, m->wte_hi, m->wte_lo}, V, E, nullptr, EPI_STORE, m->logits, nullptr, nullptr, V);
}

// One decode step for B sequences: token d_tokens[b] at position d_lens[b],
// attending over positions 0..d_lens[b] of `cache`; logits of the step into
// m->logits [B, V] and the greedy choice into d_next.          model.c:794-868
// Everything it reads from the host side is fixed at capture time, so the
// sequence can be recorded once and replayed as a graph.
// The compact copy of matrix `which` (0 qkv, 1 proj, 2 fc, 3 mlp) of layer l
// in the selected format; layer n_layer, which 0, is the tied head.
QMat qmat(const model* m, int l, int which) {
    if (m->wfmt == WF_F32) return QMat{};
    const WeightSet& s = m->sets[m->wfmt];
    return l == m->cfg.n_layer ? s.q.back() : s.q[(size_t)l * 4 + which];
}

// Builds weight format `fmt` from the loaded fp32 weights (once).
model_status build_weight_set(model* m, int fmt) {
    WeightSet& set = m->sets[fmt];
    if (set.block) return MODEL_OK;
    const size_t E = (size_t)m->cfg.n_embd, V = (size_t)m->cfg.vocab_size, L = (size_t)m->cfg.n_layer;
    struct Mtx { const float* src; size_t N, K; };
    std::vector<Mtx> mats;
    for (const Layer& y : m->base_layers) {
        mats.push_back({y.qkv_w, 3 * E, E});
        mats.push_back({y.proj_w, E, E});
        mats.push_back({y.fc_w, 4 * E, E});
        mats.push_back({y.mlp_w, E, 4 * E});
    }
    mats.push_back({m->base_wte, V, E});
    auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
    size_t bytes = 0;
    for (const Mtx& x : mats) {
        const size_t n = x.N * x.K;
        bytes += 3 * up(n * 4) + up(n * (fmt == WF_BF16 ? 2 : 1)) + (fmt == WF_INT8 ? up(x.N * 4) : 0);
    }
    char* block = nullptr;
    if (cudaMalloc(&block, bytes) != cudaSuccess) { cudaGetLastError(); return MODEL_ERR_NOMEM; }
    char* cur = block;
    auto take = [&](size_t b) { char* p = cur; cur += up(b); return p; };
    std::vector<QMat> q;
    std::vector<float*> deq, hi, lo;
    cudaError_t e = cudaSuccess;
    for (const Mtx& x : mats) {
        const size_t n = x.N * x.K;
        float* d = reinterpret_cast<float*>(take(n * 4));
        float* h = reinterpret_cast<float*>(take(n * 4));
        float* o = reinterpret_cast<float*>(take(n * 4));
        void* c = take(n * (fmt == WF_BF16 ? 2 : 1));
        float* sc = fmt == WF_INT8 ? reinterpret_cast<float*>(take(x.N * 4)) : nullptr;
        if (e == cudaSuccess)
            e = fmt == WF_BF16 ? launch_to_bf16(x.src, c, d, n, m->st)
                               : launch_quant_rows(x.src, c, sc, d, (int)x.N, (int)x.K, m->st);
        if (e == cudaSuccess) e = launch_split_hilo(d, h, o, (long long)n, m->st);
        q.push_back(QMat{fmt, c, sc});
        deq.push_back(d); hi.push_back(h); lo.push_back(o);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->st);
    if (e != cudaSuccess) {
        note_cuda(e, "building a reduced weight format", __LINE__);
        cudaGetLastError();
        cudaFree(block);
        return MODEL_ERR_DEVICE;
    }
    set.block = block;
    set.bytes = bytes;
    set.q = q;
    set.layers = m->base_layers;
    for (size_t l = 0; l < L; ++l) {
        Layer& y = set.layers[l];
        y.qkv_w = deq[4 * l]; y.qkv_hi = hi[4 * l]; y.qkv_lo = lo[4 * l];
        y.proj_w = deq[4 * l + 1]; y.proj_hi = hi[4 * l + 1]; y.proj_lo = lo[4 * l + 1];
        y.fc_w = deq[4 * l + 2]; y.fc_hi = hi[4 * l + 2]; y.fc_lo = lo[4 * l + 2];
        y.mlp_w = deq[4 * l + 3]; y.mlp_hi = hi[4 * l + 3]; y.mlp_lo = lo[4 * l + 3];
    }
    set.wte = deq.back(); set.wte_hi = hi.back(); set.wte_lo = lo.back();
    return MODEL_OK;
}

// The stream path of a decode step of B <= 8 sequences (k_decode.cu): five
// kernels per layer, LayerNorm, embedding and the attention merge folded into
// the matmuls' prologues, every matmul's weights in flight before its
// dependency wait.                                           model.c:794-868
bool use_stream(const model* m, int B) {
    return !m->stats_on && m->step_kind == TIE_STEP_STREAM && B <= kGemvRows &&
           stream_applies(B, m->cfg.n_embd, m->wfmt);
}

StreamParams stream_base(model* m, int B) {
    StreamParams p{};
    p.M = B;
    p.eps = m->cfg.layer_norm_epsilon;
    p.lens = m->d_lens;
    p.err = m->d_err;
    return p;
}

void stream_weights(StreamParams& p, const float* W, const QMat& q, const float* bias) {
    p.W = W;
    p.wt = q.wt;
    p.Wq = q.q;
    p.scale = q.s;
    p.bias = bias;
}

model_status run_decode_stream(model* m, int B, kv_cache* cache, bool advance, int32_t* out, int ld_out) {
    const int E = m->cfg.n_embd, H = m->cfg.n_head, V = m->cfg.vocab_size;
    cudaStream_t st = m->st;
    const int max_chunks = attn_decode_max_splits(cache->capacity);
    const StreamParams base = stream_base(m, B);
    int traced = 0;   // stream kernels launched so far (their trace slot)
    auto slot = [&](StreamParams& q) {
        if (m->stream_trace) q.trace = m->stream_trace + (size_t)traced * kTraceCtas * kStreamTraceEvents;
        ++traced;
    };
    for (int l = 0; l < m->cfg.n_layer; ++l) {
        const Layer& w = m->layers[l];
        const PagedKV view = layer_view(cache, l);
        // LayerNorm 1 (layer 0: of the embedding, also stored as x) + QKV + this step's K/V rows
        StreamParams p = base;
        p.epi = EPI_QKV_KV;
        p.pro = l == 0 ? STREAM_PRO_EMBED_LN : STREAM_PRO_LN;
        p.x = m->x; p.ldx = E; p.ln_g = w.ln1_w; p.ln_b = w.ln1_b;
        p.tokens = m->d_tokens; p.wte = m->wte; p.wpe = m->wpe; p.x_out = m->x; p.V = V;
        stream_weights(p, w.qkv_w, qmat(m, l, 0), w.qkv_b);
        p.y = m->qkv; p.ldy = 3 * E; p.N = 3 * E; p.K = E; p.kv = view;
        if (l == 0 && m->drill_ns) { p.stall = 1; p.wait_ns = m->drill_ns; }
        slot(p);
        LAUNCH(launch_stream_gemv(p, st));
        // attention: chunk partials
        LAUNCH(launch_attn_chunks(m->qkv, m->d_lens, B, H, view, max_chunks, m->d_part, st));
        // their merge + attention projection + residual
        p = base;
        p.epi = EPI_BIAS_RESID;
        p.pro = STREAM_PRO_MERGE;
        p.apart = m->d_part; p.H = H; p.max_chunks = max_chunks;
        stream_weights(p, w.proj_w, qmat(m, l, 1), w.proj_b);
        p.y = m->x; p.ldy = E; p.N = E; p.K = E;
        slot(p);
        LAUNCH(launch_stream_gemv(p, st));
        // LayerNorm 2 + FC + GELU
        p = base;
        p.epi = EPI_BIAS_GELU;
        p.pro = STREAM_PRO_LN;
        p.x = m->x; p.ldx = E; p.ln_g = w.ln2_w; p.ln_b = w.ln2_b;
        stream_weights(p, w.fc_w, qmat(m, l, 2), w.fc_b);
        p.y = m->ff; p.ldy = 4 * E; p.N = 4 * E; p.K = E;
        slot(p);
        LAUNCH(launch_stream_gemv(p, st));
        // MLP projection + residual
        p = base;
        p.epi = EPI_BIAS_RESID;
        p.pro = STREAM_PRO_PLAIN;
        p.x = m->ff; p.ldx = 4 * E;
        stream_weights(p, w.mlp_w, qmat(m, l, 3), w.mlp_b);
        p.y = m->x; p.ldy = E; p.N = E; p.K = 4 * E;
        slot(p);
        LAUNCH(launch_stream_gemv(p, st));
    }
    // LayerNorm f + the tied head with per-CTA greedy partials
    const QMat qh = qmat(m, m->cfg.n_layer, 0);
    StreamParams p = base;
    p.head = 1;
    p.pro = STREAM_PRO_LN;
    p.x = m->x; p.ldx = E; p.ln_g = m->lnf_w; p.ln_b = m->lnf_b;
    stream_weights(p, m->wte, qh, nullptr);
    p.y = m->logits; p.ldy = V; p.N = V; p.K = E;
    p.part_val = m->d_am_val; p.part_idx = m->d_am_idx;
    slot(p);
    LAUNCH(launch_stream_gemv(p, st));
    LAUNCH(launch_argmax_finalize(m->d_am_val, m->d_am_idx, stream_head_blocks(V, E, qh.wt, B), B, m->d_next, st));
    if (advance) LAUNCH(launch_step_advance(m->d_next, m->d_tokens, m->d_lens, out, ld_out, m->d_step, B, st));
    m->stream_traced = traced;
    return MODEL_OK;
}

model_status run_decode(model* m, int B, kv_cache* cache, bool advance, int32_t* out, int ld_out) {
    if (use_stream(m, B)) return run_decode_stream(m, B, cache, advance, out, ld_out);
    const int E = m->cfg.n_embd, H = m->cfg.n_head, V = m->cfg.vocab_size;
    const float eps = m->cfg.layer_norm_epsilon;
    cudaStream_t st = m->st;
    AttnStats* stats = m->stats_on ? m->d_stats : nullptr;
    const int max_splits = attn_decode_max_splits(cache->capacity);
    const bool small = B <= kGemvRows;
    // GEMV batches carry fp32 activations, tensor-core batches their tf32 splits
    float* xb_f = small ? m->xb : nullptr;
    float* xb_h = small ? nullptr : m->xb_hi;
    float* xb_l = small ? nullptr : m->xb_lo;
    const Mat xb{m->xb, m->xb_hi, m->xb_lo}, attn{m->attn, m->attn_hi, m->attn_lo};
    const Mat ff{m->ff, m->ff_hi, m->ff_lo};
    model_status rc;
    LAUNCH(launch_embed_decode(m->d_tokens, m->d_lens, B, m->wte, m->wpe, m->x, E, V, st));
    if (small) {
        // PDL-chained kernels: 7 per layer (k_decode.cu, k_attn.cu, k_misc.cu)
        for (int l = 0; l < m->cfg.n_layer; ++l) {
            const Layer& w = m->layers[l];
            const QMat q0 = qmat(m, l, 0), q1 = qmat(m, l, 1), q2 = qmat(m, l, 2), q3 = qmat(m, l, 3);
            const PagedKV view = layer_view(cache, l);
            // LayerNorm once per row, then the matmul over the normalised rows
            LAUNCH(launch_layernorm(m->x, w.ln1_w, w.ln1_b, m->xb, B, E, eps, st));
            LAUNCH(launch_dec_gemv(m->xb, E, nullptr, nullptr, eps, w.qkv_w, w.qkv_b, m->qkv, 3 * E, B, 3 * E, E,
                                   EPI_QKV_KV, &view, m->d_lens, st, q0.wt, q0.q, q0.s));
            LAUNCH(launch_attn_decode(m->qkv, m->d_lens, B, H, view, max_splits, m->d_part, m->attn, stats, st,
                                      nullptr, nullptr, m->d_attn_cnt, m->d_err));
            m->launches += (stats ? 2 : attn_decode_kernels(B)) - 1;  // a separate merge kernel
            LAUNCH(launch_dec_gemv(m->attn, E, nullptr, nullptr, eps, w.proj_w, w.proj_b, m->x, E, B, E, E,
                                   EPI_BIAS_RESID, nullptr, nullptr, st, q1.wt, q1.q, q1.s));
            LAUNCH(launch_layernorm(m->x, w.ln2_w, w.ln2_b, m->xb, B, E, eps, st));
            LAUNCH(launch_dec_gemv(m->xb, E, nullptr, nullptr, eps, w.fc_w, w.fc_b, m->ff, 4 * E, B, 4 * E, E,
                                   EPI_BIAS_GELU, nullptr, nullptr, st, q2.wt, q2.q, q2.s));
            LAUNCH(launch_dec_gemv(m->ff, 4 * E, nullptr, nullptr, eps, w.mlp_w, w.mlp_b, m->x, E, B, E, 4 * E,
                                   EPI_BIAS_RESID, nullptr, nullptr, st, q3.wt, q3.q, q3.s));
        }
        const QMat qh = qmat(m, m->cfg.n_layer, 0);
        LAUNCH(launch_layernorm(m->x, m->lnf_w, m->lnf_b, m->xb, B, E, eps, st));
        LAUNCH(launch_dec_head(m->xb, E, nullptr, nullptr, eps, m->wte, m->logits, V, B, V, E, m->d_am_val,
                               m->d_am_idx, st, qh.wt, qh.q, qh.s));
        LAUNCH(launch_argmax_finalize(m->d_am_val, m->d_am_idx, dec_head_blocks(V, E, qh.wt, B), B, m->d_next, st));
        if (advance)
            LAUNCH(launch_step_advance(m->d_next, m->d_tokens, m->d_lens, out, ld_out, m->d_step, B, st));
        return MODEL_OK;
    }
    for (int l = 0; l < m->cfg.n_layer; ++l) {
        const Layer& w = m->layers[l];
        const PagedKV view = layer_view(cache, l);
        LAUNCH(launch_layernorm(m->x, w.ln1_w, w.ln1_b, xb_f, B, E, eps, st, xb_h, xb_l));
        if ((rc = matmul(m, true, B, xb, E, Mat{w.qkv_w, w.qkv_hi, w.qkv_lo}, 3 * E, E, w.qkv_b, EPI_BIAS,
                         m->qkv, nullptr, nullptr, 3 * E)) != MODEL_OK)
            return rc;
        LAUNCH(launch_kv_store_decode(m->qkv, m->d_lens, B, view, st));
        LAUNCH(launch_attn_decode(m->qkv, m->d_lens, B, H, view, max_splits, m->d_part, nullptr, stats, st,
                                  m->attn_hi, m->attn_lo, m->d_attn_cnt, m->d_err));
        m->launches += (stats ? 2 : attn_decode_kernels(B)) - 1;  // a separate merge kernel
        if ((rc = matmul(m, true, B, attn, E, Mat{w.proj_w, w.proj_hi, w.proj_lo}, E, E, w.proj_b,
                         EPI_BIAS_RESID, m->x, nullptr, nullptr, E)) != MODEL_OK)
            return rc;
        LAUNCH(launch_layernorm(m->x, w.ln2_w, w.ln2_b, xb_f, B, E, eps, st, xb_h, xb_l));
        if ((rc = matmul(m, true, B, xb, E, Mat{w.fc_w, w.fc_hi, w.fc_lo}, 4 * E, E, w.fc_b, EPI_BIAS_GELU,
                         nullptr, m->ff_hi, m->ff_lo, 4 * E)) != MODEL_OK)
            return rc;
        if ((rc = matmul(m, true, B, ff, 4 * E, Mat{w.mlp_w, w.mlp_hi, w.mlp_lo}, E, 4 * E, w.mlp_b,
                         EPI_BIAS_RESID, m->x, nullptr, nullptr, E)) != MODEL_OK)
            return rc;
    }
    LAUNCH(launch_layernorm(m->x, m->lnf_w, m->lnf_b, xb_f, B, E, eps, st, xb_h, xb_l));
    if ((rc = matmul(m, true, B, xb, E, Mat{m->wte, m->wte_hi, m->wte_lo}, V, E, nullptr, EPI_STORE,
                     m->logits, nullptr, nullptr, V)) != MODEL_OK)
        return rc;
    LAUNCH(launch_argmax_rows(m->logits, V, B, V, 1, 0, m->d_next, st));
    if (advance) LAUNCH(launch_step_advance(m->d_next, m->d_tokens, m->d_lens, out, ld_out, m->d_step, B, st));
    return MODEL_OK;
}

// Runs one decode step, from a graph when statistics are off.
// Whether the persistent kernel can run a step of B sequences (fp32 weights,
// no attention statistics, a cache it can index); allocates its layer table
// and counters on first use.
bool step_applies(model* m, int B, const kv_cache* cache) {
    if (m->stats_on || m->wfmt != WF_F32 || B < 1 || B > 4) return false;
    if (!cache || cache->pages_per_seq > step_max_pages()) return false;
    int& state = m->step_state[B];
    if (state == 0) {
        int grid = 0;
        state = step_supported(B, m->cfg.n_embd, m->cfg.n_head, m->cfg.n_layer, &m->step_slots[B], &grid) ? 1 : -1;
        if (state == 1) m->step_grid = grid;
    }
    if (state != 1) return false;
    if (!m->d_step_layers) {
        const int L = m->cfg.n_layer;
        std::vector<StepLayer> table((size_t)L);
        for (int l = 0; l < L; ++l) {
            const Layer& w = m->layers[l];
            table[l] = StepLayer{w.ln1_w, w.ln1_b, w.qkv_w, w.qkv_b, w.proj_w, w.proj_b,
                                 w.ln2_w, w.ln2_b, w.fc_w, w.fc_b, w.mlp_w, w.mlp_b};
        }
        StepLayer* d = nullptr;
        unsigned* c = nullptr;
        const size_t words = step_sync_words(L);
        if (cudaMalloc(&d, table.size() * sizeof(StepLayer)) != cudaSuccess ||
            cudaMalloc(&c, words * sizeof(unsigned)) != cudaSuccess ||
            cudaMemcpy(d, table.data(), table.size() * sizeof(StepLayer), cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemset(c, 0, words * sizeof(unsigned)) != cudaSuccess) {
            cudaGetLastError();
            cudaFree(d);
            cudaFree(c);
            state = -1;
            return false;
        }
        m->d_sync = c;
        m->d_step_layers = d;
    }
    return true;
}

// A step takes the persistent kernel when it applies and the model asks for it.
bool use_step(model* m, int B, const kv_cache* cache) {
    return m->step_kind == TIE_STEP_PERSISTENT && step_applies(m, B, cache);
}

// The whole decode step of B <= 4 sequences as one persistent kernel.
model_status run_step(model* m, int B, kv_cache* cache, bool advance, int32_t* out, int ld_out,
                      unsigned long long* trace = nullptr) {
    StepParams p{};
    p.layers = m->d_step_layers;
    p.n_layer = m->cfg.n_layer; p.E = m->cfg.n_embd; p.H = m->cfg.n_head; p.V = m->cfg.vocab_size; p.M = B;
    p.eps = m->cfg.layer_norm_epsilon;
    p.scale = (float)(1.0 / std::sqrt((double)(m->cfg.n_embd / m->cfg.n_head)));
    p.wte = m->wte; p.wpe = m->wpe; p.lnf_g = m->lnf_w; p.lnf_b = m->lnf_b;
    p.k = cache->k; p.v = cache->v; p.layer_stride = cache->rows * (size_t)m->cfg.n_embd;
    p.page_table = cache->d_page_table; p.pages_per_seq = cache->pages_per_seq;
    p.max_splits = attn_decode_max_splits(cache->capacity);
    p.tokens = m->d_tokens; p.lens = m->d_lens;
    p.x = m->x; p.qkv = m->qkv; p.attn = m->attn; p.ff = m->ff;
    p.logits = m->logits; p.ldl = m->cfg.vocab_size;
    p.part = m->d_part; p.head_cnt = m->d_attn_cnt; p.sync = m->d_sync;
    p.am_val = m->d_am_val; p.am_idx = m->d_am_idx; p.next = m->d_next;
    p.advance = advance ? 1 : 0; p.out = out; p.ld_out = ld_out; p.step = m->d_step;
    p.err = m->d_err; p.slots = m->step_slots[B]; p.trace = trace;
    // about 60% of the tied head (92 MB for GPT-2) fits in L2 beside the KV cache
    p.head_prefetch = (int)std::min<size_t>((size_t)1 << 30,
                                            (size_t)m->cfg.vocab_size * m->cfg.n_embd * 4 * 6 / 10 / m->step_grid);
    LAUNCH(launch_step(p, m->step_grid, m->st));
    return MODEL_OK;
}

model_status decode_step(model* m, int B, kv_cache* cache, bool advance, int32_t* out, int ld_out) {
    if (m->stats_on) return run_decode(m, B, cache, advance, out, ld_out);
    if (m->drill_ns && use_stream(m, B)) {
        // one step run directly (not from a graph), then the drill is over
        model_status rc = run_decode(m, B, cache, advance, out, ld_out);
        m->drill_ns = 0;
        return rc;
    }
    if (use_step(m, B, cache)) return run_step(m, B, cache, advance, out, ld_out);
    const GraphKey key{B, cache, advance, out, ld_out};
    auto it = m->graphs.find(key);
    if (it == m->graphs.end()) {
        cudaGraph_t g = nullptr;
        CU(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
        const uint64_t before = m->launches;
        model_status rc = run_decode(m, B, cache, advance, out, ld_out);
        cudaError_t ce = cudaStreamEndCapture(m->st, &g);
        const uint64_t kernels = m->launches - before;
        m->launches = before;  // counted when the graph runs
        if (rc != MODEL_OK) { if (g) cudaGraphDestroy(g); return rc; }
        if (ce != cudaSuccess) { cudaGetLastError(); return MODEL_ERR_DEVICE; }
        cudaGraphExec_t ex = nullptr;
        ce = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        if (ce != cudaSuccess) { cudaGetLastError(); return MODEL_ERR_DEVICE; }
        it = m->graphs.emplace(key, GraphEntry{ex, kernels}).first;
    }
    CU(cudaGraphLaunch(it->second.exec, m->st));
    m->launches += it->second.kernels;
    return MODEL_OK;
}

model_status copy_ids_to_device(model* m, const int32_t* ids, size_t n) {
    model_status rc = ensure_rows(m, n);
    if (rc != MODEL_OK) return rc;
    CU(cudaMemcpyAsync(m->d_ids, ids, n * sizeof(int32_t), cudaMemcpyHostToDevice, m->st));
    return MODEL_OK;
}

model_status set_slot_state(model* m, size_t B, const int32_t* tokens, const int32_t* lens) {
    model_status rc = ensure_pinned(m, 2 * B);
    if (rc != MODEL_OK) return rc;
    CU(cudaStreamSynchronize(m->st));
    std::memcpy(m->h_small, tokens, B * sizeof(int32_t));
    std::memcpy(m->h_small + B, lens, B * sizeof(int32_t));
    CU(cudaMemcpyAsync(m->d_tokens, m->h_small, B * sizeof(int32_t), cudaMemcpyHostToDevice, m->st));
    CU(cudaMemcpyAsync(m->d_lens, m->h_small + B, B * sizeof(int32_t), cudaMemcpyHostToDevice, m->st));
    return MODEL_OK;
}

model_status finish(model* m) {
    CU(cudaStreamSynchronize(m->st));
    if (m->d_err) {
        int err = 0;
        CU(cudaMemcpy(&err, m->d_err, sizeof err, cudaMemcpyDeviceToHost));
        if (err) {
            std::snprintf(g_dev_err, sizeof g_dev_err, "a kernel's bounded wait expired (device error flag %d)", err);
            if (std::getenv("TIE_DEBUG")) std::fprintf(stderr, "tie_b200: %s\n", g_dev_err);
            cudaMemset(m->d_err, 0, sizeof(int));
            // a step that gave up leaves its counters wherever it stopped
            if (m->d_sync) cudaMemset(m->d_sync, 0, step_sync_words(m->cfg.n_layer) * sizeof(unsigned));
            if (m->d_attn_cnt) cudaMemset(m->d_attn_cnt, 0, m->cnt_cap * sizeof(int));
            return MODEL_ERR_DEVICE;
        }
    }
    return stats_end(m);
}

// --------------------------------------------------------------- loading --
// What a tensor must be: its rank and extents from the config, F32.
struct Expect {
    std::string name;
    int nd;
    long long d0, d1;
    size_t elems() const { return (size_t)d0 * (size_t)(nd == 2 ? d1 : 1); }
};

// Three layers of agreement are required before a tensor's bytes are read,
// and the first disagreement decides the status (the reference's load_tensor,
// model.c:287-317, refuses in this order):
//   1. the inventory record against the config: absent -> INVENTORY,
//      not F32 -> DTYPE, rank or extents -> SHAPE;
//   2. the weight file's own header against the record: absent -> INVENTORY,
//      not F32 -> DTYPE, extents, byte length or offset -> INVENTORY;
//   3. the byte length against the config's element count -> SHAPE.
model_status record_vs_config(const TensorInfo& r, const Expect& x) {
    if (r.dtype != "F32") return MODEL_ERR_DTYPE;
    if ((int)r.shape.size() != x.nd || r.shape[0] != x.d0 || (x.nd == 2 && r.shape[1] != x.d1))
        return MODEL_ERR_SHAPE;
    return MODEL_OK;
}

model_status file_vs_record(const st_tensor& t, const TensorInfo& r) {
    if (t.dtype != ST_DTYPE_F32) return MODEL_ERR_DTYPE;
    bool same = t.n_dims == (int)r.shape.size() && t.nbytes == r.nbytes && t.file_offset == r.file_offset;
    for (size_t i = 0; same && i < r.shape.size(); ++i) same = t.dims[i] == (uint64_t)r.shape[i];
    return same ? MODEL_OK : MODEL_ERR_INVENTORY;
}

model_status check_tensor(st_file* f, const Inventory& inv, const Expect& x, TensorInfo* out,
                          const st_tensor** out_t) {
    TensorInfo r;
    if (!inv.find(x.name, &r)) return MODEL_ERR_INVENTORY;
    model_status rc = record_vs_config(r, x);
    if (rc != MODEL_OK) return rc;
    const st_tensor* t = nullptr;
    if (st_find(f, x.name.c_str(), &t) != ST_OK) return MODEL_ERR_INVENTORY;
    if ((rc = file_vs_record(*t, r)) != MODEL_OK) return rc;
    if (t->nbytes != x.elems() * sizeof(float)) return MODEL_ERR_SHAPE;
    if (out) *out = r;
    if (out_t) *out_t = t;
    return MODEL_OK;
}

// Every tensor the forward pass uses, in load order.
std::vector<Expect> expected_tensors(const model_config& c) {
    const long long E = c.n_embd;
    std::vector<Expect> w = {{"wte.weight", 2, c.vocab_size, E}, {"wpe.weight", 2, c.n_ctx, E},
                             {"ln_f.weight", 1, E, 0}, {"ln_f.bias", 1, E, 0}};
    static const struct { const char* suffix; int nd; int r0, r1; } kLayer[] = {
        {"ln_1.weight", 1, 1, 0},        {"ln_1.bias", 1, 1, 0},
        {"attn.c_attn.weight", 2, 1, 3}, {"attn.c_attn.bias", 1, 3, 0},
        {"attn.c_proj.weight", 2, 1, 1}, {"attn.c_proj.bias", 1, 1, 0},
        {"ln_2.weight", 1, 1, 0},        {"ln_2.bias", 1, 1, 0},
        {"mlp.c_fc.weight", 2, 1, 4},    {"mlp.c_fc.bias", 1, 4, 0},
        {"mlp.c_proj.weight", 2, 4, 1},  {"mlp.c_proj.bias", 1, 1, 0}};
    for (int l = 0; l < c.n_layer; ++l)
        for (const auto& k : kLayer)
            w.push_back({"h." + std::to_string(l) + "." + k.suffix, k.nd, k.r0 * E, k.r1 * E});
    return w;
}

// Every tensor checked before any device work, so that a bad artifact is
// refused without touching the GPU.
model_status check_all(st_file* f, const Inventory& inv, const model_config& c) {
    for (const Expect& x : expected_tensors(c)) {
        model_status rc = check_tensor(f, inv, x, nullptr, nullptr);
        if (rc != MODEL_OK) return rc;
    }
    return MODEL_OK;
}

void record(model* m, const char* name, const TensorInfo& e, int transposed, const char* how) {
    model_tensor_record r;
    std::memset(&r, 0, sizeof r);
    std::snprintf(r.name, sizeof r.name, "%s", name);
    if (e.shape.size() == 2) std::snprintf(r.stored_shape, sizeof r.stored_shape, "%lldx%lld", e.shape[0], e.shape[1]);
    else if (!e.shape.empty()) std::snprintf(r.stored_shape, sizeof r.stored_shape, "%lld", e.shape[0]);
    std::snprintf(r.inventory_orientation, sizeof r.inventory_orientation, "%s", e.orientation.c_str());
    r.transposed_at_load = transposed;
    std::snprintf(r.reconciliation, sizeof r.reconciliation, "%s", how);
    m->records.push_back(r);
}

// The config's model shape: every value read from the artifact, none
// defaulted (model.c:345-365). Integer fields are numbers, the epsilon a
// number, the activation a string naming gelu_new.
model_status read_config(const std::string& text, model_config* cf) {
    json::Value doc;
    if (!json::parse(text.data(), text.size(), &doc) || doc.kind != json::Kind::Object) return MODEL_ERR_CONFIG;
    const json::Value* eps = doc.get("layer_norm_epsilon");
    std::string act;
    if (!field_int(doc, "n_layer", &cf->n_layer) || !field_int(doc, "n_head", &cf->n_head) ||
        !field_int(doc, "n_embd", &cf->n_embd) || !field_int(doc, "n_ctx", &cf->n_ctx) ||
        !field_int(doc, "vocab_size", &cf->vocab_size) || !eps || !eps->is_number() ||
        !field_str(doc, "activation_function", &act) || act.size() >= sizeof cf->activation_function)
        return MODEL_ERR_CONFIG;
    cf->layer_norm_epsilon = (float)eps->num;
    std::snprintf(cf->activation_function, sizeof cf->activation_function, "%s", act.c_str());
    if (cf->n_head <= 0 || cf->n_embd % cf->n_head != 0) return MODEL_ERR_CONFIG;
    cf->head_dim = cf->n_embd / cf->n_head;
    if (act != "gelu_new") return MODEL_ERR_CONFIG;
    // The kernels are written for GPT-2's head width and 16-byte rows.
    if (cf->head_dim != 64 || cf->n_embd % 4 != 0 || cf->n_layer <= 0 || cf->n_ctx <= 0 || cf->vocab_size <= 0)
        return MODEL_ERR_CONFIG;
    return MODEL_OK;
}

// The inventory must parse and must have been produced against the same model
// shape as the config (model.c:372-385).
model_status read_inventory(const std::string& text, const model_config& cf, Inventory* inv) {
    if (!inv->parse(text)) return MODEL_ERR_INVENTORY;
    const json::Value* cv = inv->config_values();
    int e = 0, l = 0, h = 0, v = 0;
    if (!cv || !field_int(*cv, "n_embd", &e) || !field_int(*cv, "n_layer", &l) || !field_int(*cv, "n_head", &h) ||
        !field_int(*cv, "vocab_size", &v))
        return MODEL_ERR_INVENTORY;
    if (e != cf.n_embd || l != cf.n_layer || h != cf.n_head || v != cf.vocab_size) return MODEL_ERR_INVENTORY;
    return MODEL_OK;
}

model_status load_impl(const char* weights_path, const char* inventory_path, const char* config_path,
                       model_cproj_reading cproj, int device, model** out) {
    if (!weights_path || !inventory_path || !config_path || !out) return MODEL_ERR_ARG;
    *out = nullptr;
    std::string cfg_text, inv_text;
    if (!json::read_file(config_path, &cfg_text)) return MODEL_ERR_OPEN;
    if (!json::read_file(inventory_path, &inv_text)) return MODEL_ERR_OPEN;

    model* m = new (std::nothrow) model();
    if (!m) return MODEL_ERR_NOMEM;
    m->cproj = cproj;
    model_status rc = MODEL_OK;
    st_file* f = nullptr;
    float* staging = nullptr;
    // pinned staging: file chunks are read into one buffer while the other's
    // copy to the device runs
    constexpr size_t kPinBytes = 32u << 20;
    void* pin[2] = {nullptr, nullptr};
    cudaEvent_t pin_done[2] = {nullptr, nullptr};
    int pin_cur = 0;
    model_config& cf = m->cfg;
    Inventory inv;
    if ((rc = read_config(cfg_text, &cf)) != MODEL_OK) goto fail;
    if ((rc = read_inventory(inv_text, cf, &inv)) != MODEL_OK) goto fail;
    if (st_open(weights_path, &f) != ST_OK) { rc = MODEL_ERR_WEIGHTS; goto fail; }
    if ((rc = check_all(f, inv, cf)) != MODEL_OK) goto fail;

    {
        if (cudaSetDevice(device) != cudaSuccess) { cudaGetLastError(); rc = MODEL_ERR_DEVICE; goto fail; }
        m->device = device;
        if (cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) != cudaSuccess) {
            cudaGetLastError();
            rc = MODEL_ERR_DEVICE;
            goto fail;
        }
        const size_t E = (size_t)cf.n_embd, V = (size_t)cf.vocab_size, L = (size_t)cf.n_layer;
        const size_t per_layer = 4 * E + 3 * E * E + 3 * E + E * E + E + 4 * E * E + 4 * E + 4 * E * E + E;
        const size_t total = V * E + (size_t)cf.n_ctx * E + 2 * E + L * per_layer;
        m->weight_bytes = total * sizeof(float);
        if (cudaMalloc(&m->d_weights, m->weight_bytes) != cudaSuccess) {
            cudaGetLastError();
            rc = MODEL_ERR_NOMEM;
            goto fail;
        }
        if (cudaMalloc(&staging, 4 * E * E * sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            rc = MODEL_ERR_NOMEM;
            goto fail;
        }
        for (int i = 0; i < 2; ++i) {
            if (cudaHostAlloc(&pin[i], kPinBytes, cudaHostAllocDefault) != cudaSuccess ||
                cudaEventCreateWithFlags(&pin_done[i], cudaEventDisableTiming) != cudaSuccess) {
                cudaGetLastError();
                rc = MODEL_ERR_NOMEM;
                goto fail;
            }
        }
        float* cursor = m->d_weights;
        auto take = [&](size_t n) { float* p = cursor; cursor += n; return p; };
        // tensor `name` (d0 x d1 row-major in the file) to dst on the device,
        // transposed to d1 x d0 when asked: chunks through the pinned buffers,
        // asynchronous copies on the model's stream
        auto fetch = [&](const char* name, int nd, size_t d0, size_t d1, TensorInfo* out, float* dst,
                         bool transpose) -> model_status {
            const st_tensor* t = nullptr;
            model_status r = check_tensor(f, inv, Expect{name, nd, (long long)d0, (long long)d1}, out, &t);
            if (r != MODEL_OK) return r;
            char* target = reinterpret_cast<char*>(transpose ? staging : dst);
            for (uint64_t off = 0; off < t->nbytes; off += kPinBytes) {
                const size_t n = (size_t)std::min<uint64_t>(kPinBytes, t->nbytes - off);
                CU(cudaEventSynchronize(pin_done[pin_cur]));
                if (st_tensor_read_range(f, t, off, pin[pin_cur], n) != ST_OK) return MODEL_ERR_WEIGHTS;
                CU(cudaMemcpyAsync(target + off, pin[pin_cur], n, cudaMemcpyHostToDevice, m->st));
                CU(cudaEventRecord(pin_done[pin_cur], m->st));
                pin_cur ^= 1;
            }
            if (transpose) CU(launch_transpose(staging, dst, (int)d0, (int)d1, m->st));
            return MODEL_OK;
        };
        TensorInfo e;
#define TRY(x) do { rc = (x); if (rc != MODEL_OK) goto fail; } while (0)
        m->wte = take(V * E);
        TRY(fetch("wte.weight", 2, V, E, &e, m->wte, false));
        record(m, "wte.weight", e, 0, "rows are tokens: the lookup table and, as stored, the tied head");
        m->wpe = take((size_t)cf.n_ctx * E);
        TRY(fetch("wpe.weight", 2, (size_t)cf.n_ctx, E, &e, m->wpe, false));
        record(m, "wpe.weight", e, 0, "rows are positions: learned absolute, as stored");
        m->lnf_w = take(E);
        TRY(fetch("ln_f.weight", 1, E, 0, &e, m->lnf_w, false));
        m->lnf_b = take(E);
        TRY(fetch("ln_f.bias", 1, E, 0, &e, m->lnf_b, false));
        m->layers.resize(L);
        for (int l = 0; l < cf.n_layer; ++l) {
            Layer& y = m->layers[l];
            char name[64];
            auto vec = [&](const char* fmt, size_t n, float** dst) -> model_status {
                std::snprintf(name, sizeof name, fmt, l);
                *dst = take(n);
                return fetch(name, 1, n, 0, nullptr, *dst, false);
            };
            // A matrix stored [in, out] in the file becomes [out, in] (K-major) on the
            // device: the layout of every matmul kernel here.
            auto mat = [&](const char* fmt, size_t din, size_t dout, bool stored_in_out,
                           float** dst) -> model_status {
                std::snprintf(name, sizeof name, fmt, l);
                *dst = take(din * dout);
                return fetch(name, 2, din, dout, &e, *dst, stored_in_out);
            };
            TRY(vec("h.%d.ln_1.weight", E, &y.ln1_w));
            TRY(vec("h.%d.ln_1.bias", E, &y.ln1_b));
            TRY(mat("h.%d.attn.c_attn.weight", E, 3 * E, true, &y.qkv_w));
            if (l == 0) record(m, "h.*.attn.c_attn.weight", e, 0,
                               "[input, output] as stored; held [output, input] on the device");
            TRY(vec("h.%d.attn.c_attn.bias", 3 * E, &y.qkv_b));
            // c_proj: the AS_STORED reading is [input, output]; the TRANSPOSED
            // reading takes the file as [output, input] (model.c:435).
            TRY(mat("h.%d.attn.c_proj.weight", E, E, cproj == MODEL_CPROJ_AS_STORED, &y.proj_w));
            if (l == 0) record(m, "h.*.attn.c_proj.weight", e, cproj == MODEL_CPROJ_TRANSPOSED,
                               cproj == MODEL_CPROJ_TRANSPOSED
                                   ? "unresolved by shape; TRANSPOSED reading, i.e. stored [output, input]"
                                   : "unresolved by shape; AS STORED reading, i.e. [input, output]");
            TRY(vec("h.%d.attn.c_proj.bias", E, &y.proj_b));
            TRY(vec("h.%d.ln_2.weight", E, &y.ln2_w));
            TRY(vec("h.%d.ln_2.bias", E, &y.ln2_b));
            TRY(mat("h.%d.mlp.c_fc.weight", E, 4 * E, true, &y.fc_w));
            if (l == 0) record(m, "h.*.mlp.c_fc.weight", e, 0,
                               "[input, output] as stored; held [output, input] on the device");
            TRY(vec("h.%d.mlp.c_fc.bias", 4 * E, &y.fc_b));
            TRY(mat("h.%d.mlp.c_proj.weight", 4 * E, E, true, &y.mlp_w));
            if (l == 0) record(m, "h.*.mlp.c_proj.weight", e, 0,
                               "[input, output] as stored; held [output, input] on the device");
            TRY(vec("h.%d.mlp.c_proj.bias", E, &y.mlp_b));
        }
        // every copy and transpose on the model's stream has landed
        CU(cudaStreamSynchronize(m->st));
        // tf32 splits of every matrix, for the tensor-core matmul
        {
            const size_t mats = V * E + L * (3 * E * E + E * E + 4 * E * E + 4 * E * E);
            m->split_bytes = 2 * mats * sizeof(float);
            if (cudaMalloc(&m->d_split, m->split_bytes) != cudaSuccess) {
                cudaGetLastError();
                rc = MODEL_ERR_NOMEM;
                goto fail;
            }
            float* sc = m->d_split;
            auto split = [&](const float* src, size_t n, float** hi, float** lo) -> model_status {
                *hi = sc;
                *lo = sc + n;
                sc += 2 * n;
                CU(launch_split_hilo(src, *hi, *lo, (long long)n, nullptr));
                return MODEL_OK;
            };
            TRY(split(m->wte, V * E, &m->wte_hi, &m->wte_lo));
            for (auto& y : m->layers) {
                TRY(split(y.qkv_w, 3 * E * E, &y.qkv_hi, &y.qkv_lo));
                TRY(split(y.proj_w, E * E, &y.proj_hi, &y.proj_lo));
                TRY(split(y.fc_w, 4 * E * E, &y.fc_hi, &y.fc_lo));
                TRY(split(y.mlp_w, 4 * E * E, &y.mlp_hi, &y.mlp_lo));
            }
            m->base_layers = m->layers;
            m->base_wte = m->wte; m->base_wte_hi = m->wte_hi; m->base_wte_lo = m->wte_lo;
            if (cudaDeviceSynchronize() != cudaSuccess) {
                cudaGetLastError();
                rc = MODEL_ERR_DEVICE;
                goto fail;
            }
        }
#undef TRY
    }
    cudaFree(staging);
    for (int i = 0; i < 2; ++i) {
        if (pin_done[i]) cudaEventDestroy(pin_done[i]);
        if (pin[i]) cudaFreeHost(pin[i]);
    }
    st_close(f);
    *out = m;
    return MODEL_OK;
fail:
    if (m && m->st) cudaStreamSynchronize(m->st);   // no copy still reads a pinned buffer
    cudaFree(staging);
    for (int i = 0; i < 2; ++i) {
        if (pin_done[i]) cudaEventDestroy(pin_done[i]);
        if (pin[i]) cudaFreeHost(pin[i]);
    }
    if (f) st_close(f);
    model_free(m);
    return rc;
}

}  // namespace

// ================================================================== the ABI ==
extern "C" {

const char* tie_last_device_error(void) { return g_dev_err; }

const char* model_strerror(model_status s) {
    switch (s) {
        case MODEL_OK: return "ok";
        case MODEL_ERR_OPEN: return "an artifact could not be opened";
        case MODEL_ERR_CONFIG: return "config.json is missing a field or names an unsupported architecture";
        case MODEL_ERR_INVENTORY: return "the inventory disagrees with the weight file";
        case MODEL_ERR_WEIGHTS: return "the weight file failed to open, parse or read";
        case MODEL_ERR_SHAPE: return "a tensor's shape contradicts the config";
        case MODEL_ERR_DTYPE: return "a tensor is not F32";
        case MODEL_ERR_RANGE: return "a token id or position is out of range";
        case MODEL_ERR_CAPACITY: return "a caller-owned buffer or the cache is too small";
        case MODEL_ERR_NOMEM: return "allocation failed";
        case MODEL_ERR_ARG: return "a null or unusable argument";
        case MODEL_ERR_DEVICE: return "a CUDA call failed";
    }
    return "unknown";
}

model_status model_load(const char* weights_path, const char* inventory_path, const char* config_path,
                        model_cproj_reading cproj_reading, model** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); dev = 0; }
    return load_impl(weights_path, inventory_path, config_path, cproj_reading, dev, out);
}

model_status model_load_on_device(const char* weights_path, const char* inventory_path,
                                  const char* config_path, model_cproj_reading cproj_reading,
                                  int device, model** out) {
    return load_impl(weights_path, inventory_path, config_path, cproj_reading, device, out);
}

void model_free(model* m) {
    if (!m) return;
    if (m->st) cudaStreamSynchronize(m->st);
    drop_graphs(m);
    cudaFree(m->d_weights);
    cudaFree(m->d_split);
    cudaFree(m->x);  // the activation block (x, xb, qkv, attn, ff and their splits)
    cudaFree(m->d_err);
    cudaFree(m->logits); cudaFree(m->d_ids);
    cudaFree(m->d_tokens); cudaFree(m->d_lens); cudaFree(m->d_next); cudaFree(m->d_step);
    cudaFree(m->d_out); cudaFree(m->d_part); cudaFree(m->d_attn_cnt); cudaFree(m->d_am_val); cudaFree(m->d_am_idx);
    cudaFree(m->d_stats);
    cudaFree(m->d_step_layers); cudaFree(m->d_sync);
    cudaFree(m->sets[1].block); cudaFree(m->sets[2].block);
    if (m->h_small) cudaFreeHost(m->h_small);
    kv_cache_destroy(m->kv);
    kv_cache_destroy(m->pool);
    if (m->st) cudaStreamDestroy(m->st);
    cudaGetLastError();
    delete m;
}

const model_config* model_config_of(const model* m) { return m ? &m->cfg : nullptr; }
model_cproj_reading model_cproj_reading_of(const model* m) { return m ? m->cproj : MODEL_CPROJ_AS_STORED; }
size_t model_tensor_record_count(const model* m) { return m ? m->records.size() : 0; }
const model_tensor_record* model_tensor_record_at(const model* m, size_t i) {
    return (m && i < m->records.size()) ? &m->records[i] : nullptr;
}

// The forward pass has no substitutable CPU matmul; the choice is recorded and
// the engine's own kernels keep running (model_gemm_of reports them).
void model_set_gemm(model* m, const gemm_impl* impl) { if (m && impl) m->gemm_choice = impl; }
const gemm_impl* model_gemm_of(const model* m) { return m ? &gemm_impl_sm100a : nullptr; }

void model_set_decode_path(model* m, model_decode_path p) {
    if (m && (p == MODEL_PATH_NOCACHE || p == MODEL_PATH_CACHE)) m->path = p;
}
model_decode_path model_decode_path_of(const model* m) { return m ? m->path : MODEL_PATH_NOCACHE; }

model_status model_reserve(model* m, size_t T) {
    if (!m) return MODEL_ERR_ARG;
    if (T == 0) T = 1;
    model_status rc = ensure_rows(m, T);
    if (rc != MODEL_OK) return rc;
    rc = ensure_logits(m, T);
    if (rc != MODEL_OK) return rc;
    return ensure_slots(m, 1, m->cfg.n_ctx);
}

model_status model_kv_reserve(model* m, size_t capacity) {
    if (!m) return MODEL_ERR_ARG;
    if (capacity == 0) return MODEL_ERR_ARG;
    if ((int)capacity > m->cfg.n_ctx) return MODEL_ERR_RANGE;
    if (m->kv && kv_cache_capacity(m->kv) >= (int)capacity) return MODEL_OK;
    kv_cache* fresh = nullptr;
    kv_status ks = kv_cache_create(m->cfg.n_layer, m->cfg.n_embd, (int)capacity, &fresh);
    if (ks == KV_ERR_NOMEM) return MODEL_ERR_NOMEM;
    if (ks != KV_OK) return MODEL_ERR_ARG;
    drop_graphs(m);
    kv_cache_destroy(m->kv);
    m->kv = fresh;
    return MODEL_OK;
}

size_t model_kv_footprint_bytes(const model* m) { return m ? kv_cache_footprint_bytes(m->kv) : 0u; }
int model_kv_capacity(const model* m) { return m ? kv_cache_capacity(m->kv) : 0; }
int model_kv_length(const model* m) { return m ? kv_cache_length(m->kv) : 0; }
const kv_cache* model_kv_cache_of(const model* m) { return m ? m->kv : nullptr; }

model_status model_kv_set_length(model* m, int length) {
    if (!m || !m->kv) return MODEL_ERR_ARG;
    kv_status ks = kv_cache_set_length(m->kv, length);
    if (ks == KV_ERR_CAPACITY) return MODEL_ERR_CAPACITY;
    return ks == KV_OK ? MODEL_OK : MODEL_ERR_ARG;
}

const float* model_token_embedding(const model* m) { return m ? m->wte : nullptr; }
const float* model_head_weight(const model* m) { return m ? m->wte : nullptr; }

void model_collect_attn_stats(model* m, int enable) {
    if (!m) return;
    m->stats_on = enable != 0;
    m->rs_min = m->rs_max = 0.0;
    m->rs_rows = 0;
}

void model_attn_rowsum_range(const model* m, double* lo, double* hi, size_t* rows) {
    if (lo) *lo = m ? m->rs_min : 0.0;
    if (hi) *hi = m ? m->rs_max : 0.0;
    if (rows) *rows = m ? m->rs_rows : 0;
}

// model.c:920-925: a strict '>' scan of a HOST buffer; lowest index wins ties.
int32_t model_argmax(const float* v, size_t n) {
    int32_t best = 0;
    for (size_t i = 1; i < n; ++i) if (v[i] > v[best]) best = (int32_t)i;
    return best;
}

// model.c:593-603, computed by the engine's LayerNorm kernel with unit gain and
// zero shift (x * 1 + 0 leaves the normalised value unchanged). Host arrays in
// and out; NaN is written if no device is usable.
void model_layernorm_normalize(const float* x, int n, float eps, float* out) {
    if (!x || !out || n <= 0) return;
    float* d = nullptr;
    std::vector<float> ones((size_t)n, 1.0f);
    bool ok = cudaMalloc(&d, (size_t)n * 4 * 4) == cudaSuccess;
    if (ok) {
        float *dx = d, *dy = d + n, *dg = d + 2 * (size_t)n, *db = d + 3 * (size_t)n;
        ok = cudaMemcpy(dx, x, (size_t)n * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemcpy(dg, ones.data(), (size_t)n * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemset(db, 0, (size_t)n * 4) == cudaSuccess &&
             launch_layernorm(dx, dg, db, dy, 1, n, eps, nullptr) == cudaSuccess &&
             cudaMemcpy(out, dy, (size_t)n * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
    }
    cudaFree(d);
    if (!ok) {
        cudaGetLastError();
        for (int i = 0; i < n; ++i) out[i] = NAN;
    }
}

model_status tie_attention_prefill(const float* qkv, int n_seq, int T, int n_head, float* out) {
    if (!qkv || !out || n_seq <= 0 || T <= 0 || n_head <= 0) return MODEL_ERR_ARG;
    const size_t E = (size_t)n_head * 64, rows = (size_t)n_seq * T;
    float *dq = nullptr, *dout = nullptr;
    int* derr = nullptr;
    int herr = 0;
    bool ok = cudaMalloc(&dq, rows * 3 * E * 4) == cudaSuccess && cudaMalloc(&dout, rows * E * 4) == cudaSuccess &&
              cudaMalloc(&derr, sizeof(int)) == cudaSuccess && cudaMemset(derr, 0, sizeof(int)) == cudaSuccess &&
              cudaMemcpy(dq, qkv, rows * 3 * E * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              launch_attn_prefill(dq, n_seq, T, n_head, dout, nullptr, nullptr, nullptr, nullptr, derr) ==
                  cudaSuccess &&
              cudaMemcpy(out, dout, rows * E * 4, cudaMemcpyDeviceToHost) == cudaSuccess &&
              cudaMemcpy(&herr, derr, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess;
    if (!ok) {
        note_cuda(cudaGetLastError(), "tie_attention_prefill", __LINE__);
        cudaGetLastError();
    }
    cudaFree(dq);
    cudaFree(dout);
    cudaFree(derr);
    return ok && herr == 0 ? MODEL_OK : MODEL_ERR_DEVICE;
}

// ---------------------------------------------------------------- prefill --
model_status model_prefill(model* m, const int32_t* ids, size_t T, float* logits, size_t cap) {
    if (!m || !ids || !logits) return MODEL_ERR_ARG;
    if (cap < T * (size_t)m->cfg.vocab_size) return MODEL_ERR_CAPACITY;
    model_status rc = model_reserve(m, T);
    if (rc != MODEL_OK) return rc;
    // forward_blocks' refusals, all before any launch (model.c:660-668)
    const bool use_cache = m->path == MODEL_PATH_CACHE;
    if (T == 0) return MODEL_ERR_ARG;
    if ((int)T > m->cfg.n_ctx) return MODEL_ERR_RANGE;
    for (size_t t = 0; t < T; ++t)
        if (ids[t] < 0 || ids[t] >= m->cfg.vocab_size) return MODEL_ERR_RANGE;
    if (use_cache) {
        if (!m->kv) return MODEL_ERR_ARG;
        if ((int)T > kv_cache_capacity(m->kv)) return MODEL_ERR_CAPACITY;
    }
    if ((rc = stats_begin(m)) != MODEL_OK) return rc;
    if ((rc = copy_ids_to_device(m, ids, T)) != MODEL_OK) return rc;
    if ((rc = run_prefill(m, 1, (int)T, use_cache ? m->kv : nullptr, 0)) != MODEL_OK) return rc;
    const int V = m->cfg.vocab_size;
    // the tied head at every position (model.c:778-780)
    if ((rc = prefill_head(m, (int)T, 0, 1)) != MODEL_OK) return rc;
    CU(cudaMemcpyAsync(logits, m->logits, T * (size_t)V * sizeof(float), cudaMemcpyDeviceToHost, m->st));
    if ((rc = finish(m)) != MODEL_OK) return rc;
    if (use_cache) kv_cache_set_length(m->kv, (int)T);
    return MODEL_OK;
}

// ----------------------------------------------------------------- decode --
static model_status cached_step(model* m, const int32_t* ids, size_t T, float* logits, int32_t* next) {
    model_status rc = model_reserve(m, T);
    if (rc != MODEL_OK) return rc;
    const int32_t id = ids[T - 1];
    if (id < 0 || id >= m->cfg.vocab_size) return MODEL_ERR_RANGE;
    if ((rc = ensure_slots(m, 1, m->kv->capacity)) != MODEL_OK) return rc;
    if ((rc = stats_begin(m)) != MODEL_OK) return rc;
    const int32_t len = (int32_t)(T - 1);
    if ((rc = set_slot_state(m, 1, &id, &len)) != MODEL_OK) return rc;
    if ((rc = decode_step(m, 1, m->kv, false, nullptr, 0)) != MODEL_OK) return rc;
    if (logits)
        CU(cudaMemcpyAsync(logits, m->logits, (size_t)m->cfg.vocab_size * sizeof(float),
                           cudaMemcpyDeviceToHost, m->st));
    if (next) CU(cudaMemcpyAsync(m->h_small, m->d_next, sizeof(int32_t), cudaMemcpyDeviceToHost, m->st));
    if ((rc = finish(m)) != MODEL_OK) return rc;
    if (next) *next = m->h_small[0];
    kv_cache_set_length(m->kv, (int)T);
    return MODEL_OK;
}

model_status model_decode_step_cached(model* m, const int32_t* ids, size_t T, float* logits, size_t cap) {
    if (!m || !ids || !logits) return MODEL_ERR_ARG;
    if (cap < (size_t)m->cfg.vocab_size) return MODEL_ERR_CAPACITY;
    if (T == 0) return MODEL_ERR_ARG;
    if ((int)T > m->cfg.n_ctx) return MODEL_ERR_RANGE;
    if (!m->kv) return MODEL_ERR_ARG;
    if ((int)T > kv_cache_capacity(m->kv)) return MODEL_ERR_CAPACITY;
    if (kv_cache_length(m->kv) != (int)(T - 1)) return MODEL_ERR_ARG;
    return cached_step(m, ids, T, logits, nullptr);
}

model_status model_decode_step_greedy(model* m, const int32_t* ids, size_t T, int32_t* next) {
    if (!m || !ids || !next) return MODEL_ERR_ARG;
    if (T == 0) return MODEL_ERR_ARG;
    if ((int)T > m->cfg.n_ctx) return MODEL_ERR_RANGE;
    if (!m->kv) return MODEL_ERR_ARG;
    if ((int)T > kv_cache_capacity(m->kv)) return MODEL_ERR_CAPACITY;
    if (kv_cache_length(m->kv) != (int)(T - 1)) return MODEL_ERR_ARG;
    return cached_step(m, ids, T, nullptr, next);
}

model_status model_decode_step(model* m, const int32_t* ids, size_t T, float* logits, size_t cap) {
    if (!m || !ids || !logits) return MODEL_ERR_ARG;
    if (m->path == MODEL_PATH_CACHE) return model_decode_step_cached(m, ids, T, logits, cap);
    if (cap < (size_t)m->cfg.vocab_size) return MODEL_ERR_CAPACITY;
    model_status rc = model_reserve(m, T);
    if (rc != MODEL_OK) return rc;
    if (T == 0) return MODEL_ERR_ARG;
    if ((int)T > m->cfg.n_ctx) return MODEL_ERR_RANGE;
    for (size_t t = 0; t < T; ++t)
        if (ids[t] < 0 || ids[t] >= m->cfg.vocab_size) return MODEL_ERR_RANGE;
    if ((rc = stats_begin(m)) != MODEL_OK) return rc;
    if ((rc = copy_ids_to_device(m, ids, T)) != MODEL_OK) return rc;
    if ((rc = run_prefill(m, 1, (int)T, nullptr, 0)) != MODEL_OK) return rc;
    const int V = m->cfg.vocab_size;
    // the head at the last position only, with prefill's kernel (model.c:913-916)
    if ((rc = prefill_head(m, 1, T - 1, 1)) != MODEL_OK) return rc;
    CU(cudaMemcpyAsync(logits, m->logits, (size_t)V * sizeof(float), cudaMemcpyDeviceToHost, m->st));
    return finish(m);
}

// ----------------------------------------------------------------- batches --
int model_device(const model* m) { return m ? m->device : -1; }
void* model_stream(const model* m) { return m ? (void*)m->st : nullptr; }
size_t model_weight_device_bytes(const model* m) {
    return m ? m->weight_bytes + m->split_bytes + m->sets[1].bytes + m->sets[2].bytes : 0;
}
uint64_t model_kernel_launches(const model* m) { return m ? m->launches : 0; }

// Pages covering positions [0, length) for the pool's sequences [0, n_seq),
// assigned from the pool's free pages, the device table updated on the model's
// stream (before the kernels that follow).
static model_status map_pages(model* m, size_t n_seq, size_t length) {
    const kv_status ks = kv_pool_map(m->pool, (int)n_seq, (int)length, m->st);
    if (ks == KV_OK) return MODEL_OK;
    if (ks == KV_ERR_CAPACITY) return MODEL_ERR_CAPACITY;
    if (ks == KV_ERR_NOMEM) {
        note_cuda(cudaErrorMemoryAllocation, "page table update", __LINE__);
        return MODEL_ERR_DEVICE;
    }
    return MODEL_ERR_ARG;
}

model_status model_batch_reserve(model* m, size_t n_seq, size_t capacity) {
    return model_batch_reserve_pages(m, n_seq, capacity, 0);
}

model_status model_batch_reserve_pages(model* m, size_t n_seq, size_t capacity, size_t n_pages) {
    if (!m || n_seq == 0 || capacity == 0) return MODEL_ERR_ARG;
    if ((int)capacity > m->cfg.n_ctx) return MODEL_ERR_RANGE;
    if (n_seq > 1024) return MODEL_ERR_ARG;
    const size_t per_seq = (capacity + KV_CACHE_PAGE_ROWS - 1) / KV_CACHE_PAGE_ROWS;
    if (n_pages > n_seq * per_seq) return MODEL_ERR_ARG;
    const int want_pages = (int)(n_pages ? n_pages : n_seq * per_seq);
    // a new pool unless the current one covers the request: as many sequences,
    // as long, and exactly n_pages pages (n_pages given) or at least a full
    // reservation's pages (n_pages 0)
    if (!m->pool || m->pool->n_seq < (int)n_seq || m->pool->capacity < (int)capacity ||
        (n_pages ? m->pool->pages.n_pages() != want_pages : m->pool->pages.n_pages() < want_pages)) {
        kv_cache* fresh = nullptr;
        kv_status ks = kv_pool_create(m->cfg.n_layer, m->cfg.n_embd, (int)n_seq, (int)capacity, (int)n_pages,
                                      &fresh);
        if (ks != KV_OK) return ks == KV_ERR_NOMEM ? MODEL_ERR_NOMEM : MODEL_ERR_ARG;
        drop_graphs(m);
        kv_cache_destroy(m->pool);
        m->pool = fresh;
    }
    model_status rc = ensure_rows(m, n_seq * capacity);
    if (rc != MODEL_OK) return rc;
    rc = ensure_slots(m, n_seq, m->pool->capacity);
    if (rc != MODEL_OK) return rc;
    return ensure_logits(m, n_seq);
}

model_status model_batch_release(model* m, size_t seq) {
    if (!m || !m->pool || seq >= (size_t)m->pool->n_seq) return MODEL_ERR_ARG;
    return kv_pool_release(m->pool, (int)seq) == KV_OK ? MODEL_OK : MODEL_ERR_ARG;
}

size_t model_batch_free_pages(const model* m) {
    return m && m->pool ? (size_t)m->pool->pages.free_pages() : 0;
}

static model_status batch_prefill_impl(model* m, size_t n_seq, size_t T, float* logits_host,
                                       int32_t* next_host, bool host_ids, const int32_t* ids) {
    const int V = m->cfg.vocab_size;
    model_status rc;
    if (host_ids) {
        if ((rc = copy_ids_to_device(m, ids, n_seq * T)) != MODEL_OK) return rc;
    } else {
        CU(cudaMemcpyAsync(m->d_ids, ids, n_seq * T * sizeof(int32_t), cudaMemcpyDeviceToDevice, m->st));
    }
    if ((rc = map_pages(m, n_seq, T)) != MODEL_OK) return rc;
    if ((rc = run_prefill(m, (int)n_seq, (int)T, m->pool, 0)) != MODEL_OK) return rc;
    if (logits_host) {
        if ((rc = ensure_logits(m, n_seq * T)) != MODEL_OK) return rc;
        if ((rc = prefill_head(m, (int)(n_seq * T), 0, 1)) != MODEL_OK) return rc;
        CU(cudaMemcpyAsync(logits_host, m->logits, n_seq * T * (size_t)V * sizeof(float),
                           cudaMemcpyDeviceToHost, m->st));
        LAUNCH(launch_argmax_rows(m->logits, V, (int)n_seq, V, (int)T, (int)T - 1, m->d_next, m->st));
    } else {
        // head only at each sequence's last position: rows (T-1) + s*T of xb
        if ((rc = prefill_head(m, (int)n_seq, T - 1, (int)T)) != MODEL_OK) return rc;
        LAUNCH(launch_argmax_rows(m->logits, V, (int)n_seq, V, 1, 0, m->d_next, m->st));
    }
    (void)next_host;
    return MODEL_OK;
}

model_status model_prefill_batch(model* m, const int32_t* ids, size_t n_seq, size_t T, float* logits,
                                 size_t cap, int32_t* next_ids) {
    if (!m || !ids || n_seq == 0 || T == 0) return MODEL_ERR_ARG;
    if (!m->pool || (int)n_seq > m->pool->n_seq) return MODEL_ERR_ARG;
    if ((int)T > m->pool->capacity) return MODEL_ERR_CAPACITY;
    if (logits && cap < n_seq * T * (size_t)m->cfg.vocab_size) return MODEL_ERR_CAPACITY;
    for (size_t i = 0; i < n_seq * T; ++i)
        if (ids[i] < 0 || ids[i] >= m->cfg.vocab_size) return MODEL_ERR_RANGE;
    model_status rc = ensure_rows(m, n_seq * T);
    if (rc != MODEL_OK) return rc;
    if ((rc = stats_begin(m)) != MODEL_OK) return rc;
    if ((rc = batch_prefill_impl(m, n_seq, T, logits, next_ids, true, ids)) != MODEL_OK) return rc;
    if (next_ids)
        CU(cudaMemcpyAsync(next_ids, m->d_next, n_seq * sizeof(int32_t), cudaMemcpyDeviceToHost, m->st));
    if ((rc = finish(m)) != MODEL_OK) return rc;
    m->pool->length = (int)T;
    return MODEL_OK;
}

model_status model_decode_step_batch(model* m, const int32_t* ids, size_t n_seq, float* logits,
                                     size_t cap, int32_t* next_ids) {
    if (!m || !ids || n_seq == 0) return MODEL_ERR_ARG;
    if (!m->pool || (int)n_seq > m->pool->n_seq) return MODEL_ERR_ARG;
    if (logits && cap < n_seq * (size_t)m->cfg.vocab_size) return MODEL_ERR_CAPACITY;
    for (size_t i = 0; i < n_seq; ++i)
        if (ids[i] < 0 || ids[i] >= m->cfg.vocab_size) return MODEL_ERR_RANGE;
    if (m->pool->length + 1 > m->pool->capacity) return MODEL_ERR_CAPACITY;
    model_status rc = ensure_slots(m, n_seq, m->pool->capacity);
    if (rc != MODEL_OK) return rc;
    if ((rc = stats_begin(m)) != MODEL_OK) return rc;
    std::vector<int32_t> lens(n_seq, (int32_t)m->pool->length);
    if ((rc = set_slot_state(m, n_seq, ids, lens.data())) != MODEL_OK) return rc;
    if ((rc = map_pages(m, n_seq, (size_t)m->pool->length + 1)) != MODEL_OK) return rc;
    if ((rc = decode_step(m, (int)n_seq, m->pool, false, nullptr, 0)) != MODEL_OK) return rc;
    if (logits)
        CU(cudaMemcpyAsync(logits, m->logits, n_seq * (size_t)m->cfg.vocab_size * sizeof(float),
                           cudaMemcpyDeviceToHost, m->st));
    if (next_ids)
        CU(cudaMemcpyAsync(next_ids, m->d_next, n_seq * sizeof(int32_t), cudaMemcpyDeviceToHost, m->st));
    if ((rc = finish(m)) != MODEL_OK) return rc;
    m->pool->length += 1;
    return MODEL_OK;
}

static model_status generate_impl(model* m, const int32_t* prompts, size_t n_seq, size_t T, size_t n_new,
                                  int32_t* out_ids, bool host) {
    if (!m || !prompts || !out_ids || n_seq == 0 || T == 0 || n_new == 0) return MODEL_ERR_ARG;
    if (!m->pool || (int)n_seq > m->pool->n_seq) return MODEL_ERR_ARG;
    if (T + n_new - 1 > (size_t)m->pool->capacity) return MODEL_ERR_CAPACITY;
    if (host)
        for (size_t i = 0; i < n_seq * T; ++i)
            if (prompts[i] < 0 || prompts[i] >= m->cfg.vocab_size) return MODEL_ERR_RANGE;
    model_status rc = ensure_rows(m, n_seq * T);
    if (rc != MODEL_OK) return rc;
    if ((rc = ensure_slots(m, n_seq, m->pool->capacity)) != MODEL_OK) return rc;
    int32_t* d_out = out_ids;
    if (host) {
        size_t cap = m->out_cap;
        if ((rc = grow(&m->d_out, &cap, n_seq * n_new)) != MODEL_OK) return rc;
        m->out_cap = cap;
        d_out = m->d_out;
    }
    if ((rc = stats_begin(m)) != MODEL_OK) return rc;
    if ((rc = batch_prefill_impl(m, n_seq, T, nullptr, nullptr, host, prompts)) != MODEL_OK) return rc;
    // The prefill's greedy choice is new token 0. One step_advance records it,
    // makes it the next input and moves every length from T - 1 to T; each
    // decode-step graph then ends with the same advance.
    if ((rc = ensure_pinned(m, n_seq)) != MODEL_OK) return rc;
    CU(cudaStreamSynchronize(m->st));
    for (size_t i = 0; i < n_seq; ++i) m->h_small[i] = (int32_t)T - 1;
    CU(cudaMemcpyAsync(m->d_lens, m->h_small, n_seq * sizeof(int32_t), cudaMemcpyHostToDevice, m->st));
    CU(cudaMemsetAsync(m->d_step, 0, sizeof(int32_t), m->st));
    LAUNCH(launch_step_advance(m->d_next, m->d_tokens, m->d_lens, d_out, (int)n_new, m->d_step, (int)n_seq, m->st));
    // step g writes position T + g - 1 and reads 0 .. T + g - 1: its pages are
    // assigned before it is launched (a new page every 16 steps)
    for (size_t g = 1; g < n_new; ++g) {
        if ((rc = map_pages(m, n_seq, T + g)) != MODEL_OK) return rc;
        if ((rc = decode_step(m, (int)n_seq, m->pool, true, d_out, (int)n_new)) != MODEL_OK) return rc;
    }
    if (host)
        CU(cudaMemcpyAsync(out_ids, d_out, n_seq * n_new * sizeof(int32_t), cudaMemcpyDeviceToHost, m->st));
    m->pool->length = (int)(T + n_new - 1);
    if (host) return finish(m);
    return MODEL_OK;
}

model_status model_generate_greedy(model* m, const int32_t* prompts, size_t n_seq, size_t n_prompt,
                                   size_t n_new, int32_t* out_ids) {
    return generate_impl(m, prompts, n_seq, n_prompt, n_new, out_ids, true);
}

model_status model_generate_greedy_device(model* m, const int32_t* d_prompts, size_t n_seq,
                                          size_t n_prompt, size_t n_new, int32_t* d_out_ids) {
    return generate_impl(m, d_prompts, n_seq, n_prompt, n_new, d_out_ids, false);
}

model_status model_step_trace(model* m, size_t rows, size_t context, uint64_t* out, size_t cap,
                              size_t* per_cta, size_t* n_cta) {
    if (!m || !per_cta || !n_cta || rows == 0 || rows > 4 || context == 0) return MODEL_ERR_ARG;
    if (!m->pool || (int)rows > m->pool->n_seq || (int)context > m->pool->capacity) return MODEL_ERR_CAPACITY;
    model_status rc = ensure_slots(m, rows, m->pool->capacity);
    if (rc != MODEL_OK) return rc;
    if (!step_applies(m, (int)rows, m->pool)) return MODEL_ERR_ARG;
    const size_t ev = (size_t)step_trace_events(m->cfg.n_layer), G = (size_t)m->step_grid;
    *per_cta = ev;
    *n_cta = G;
    if (!out || cap < ev * G) return MODEL_ERR_CAPACITY;
    std::vector<int32_t> lens(rows, (int32_t)context - 1), toks(rows, 1);
    if ((rc = set_slot_state(m, rows, toks.data(), lens.data())) != MODEL_OK) return rc;
    if ((rc = map_pages(m, rows, context)) != MODEL_OK) return rc;
    unsigned long long* d = nullptr;
    CU(cudaMalloc(&d, ev * G * sizeof(unsigned long long)));
    CU(cudaMemsetAsync(d, 0, ev * G * sizeof(unsigned long long), m->st));
    rc = run_step(m, (int)rows, m->pool, false, nullptr, 0);  // warm
    if (rc == MODEL_OK) rc = run_step(m, (int)rows, m->pool, false, nullptr, 0, d);
    if (rc == MODEL_OK && cudaMemcpyAsync(out, d, ev * G * sizeof(unsigned long long), cudaMemcpyDeviceToHost,
                                          m->st) != cudaSuccess)
        rc = MODEL_ERR_DEVICE;
    if (rc == MODEL_OK) rc = finish(m);
    cudaStreamSynchronize(m->st);
    cudaFree(d);
    return rc;
}

model_status model_set_weight_format(model* m, int fmt) {
    if (!m || fmt < TIE_WEIGHTS_F32 || fmt > TIE_WEIGHTS_INT8) return MODEL_ERR_ARG;
    if (fmt == m->wfmt) return MODEL_OK;
    if (fmt != WF_F32) {
        model_status rc = build_weight_set(m, fmt);
        if (rc != MODEL_OK) return rc;
    }
    CU(cudaStreamSynchronize(m->st));
    drop_graphs(m);
    if (fmt == WF_F32) {
        m->layers = m->base_layers;
        m->wte = m->base_wte; m->wte_hi = m->base_wte_hi; m->wte_lo = m->base_wte_lo;
    } else {
        const WeightSet& s = m->sets[fmt];
        m->layers = s.layers;
        m->wte = s.wte; m->wte_hi = s.wte_hi; m->wte_lo = s.wte_lo;
    }
    m->wfmt = fmt;
    return MODEL_OK;
}

int model_weight_format(const model* m) { return m ? m->wfmt : -1; }

model_status model_stream_trace(model* m, size_t rows, size_t context, uint64_t* out, size_t cap,
                                size_t* per_kernel, size_t* n_kernels) {
    if (!m || !per_kernel || !n_kernels || rows == 0 || rows > (size_t)kGemvRows || context == 0) return MODEL_ERR_ARG;
    if (!m->pool || (int)rows > m->pool->n_seq || (int)context > m->pool->capacity) return MODEL_ERR_CAPACITY;
    if (!use_stream(m, (int)rows)) return MODEL_ERR_ARG;
    const size_t kernels = 4 * (size_t)m->cfg.n_layer + 1, per = (size_t)kTraceCtas * kStreamTraceEvents;
    *per_kernel = per;
    *n_kernels = kernels;
    if (!out || cap < per * kernels) return MODEL_ERR_CAPACITY;
    model_status rc = ensure_slots(m, rows, m->pool->capacity);
    if (rc != MODEL_OK) return rc;
    std::vector<int32_t> lens(rows, (int32_t)context - 1), toks(rows, 1);
    if ((rc = set_slot_state(m, rows, toks.data(), lens.data())) != MODEL_OK) return rc;
    if ((rc = map_pages(m, rows, context)) != MODEL_OK) return rc;
    unsigned long long* d = nullptr;
    CU(cudaMalloc(&d, per * kernels * sizeof(unsigned long long)));
    CU(cudaMemsetAsync(d, 0, per * kernels * sizeof(unsigned long long), m->st));
    rc = run_decode_stream(m, (int)rows, m->pool, false, nullptr, 0);   // warm
    if (rc == MODEL_OK) {
        m->stream_trace = d;
        rc = run_decode_stream(m, (int)rows, m->pool, false, nullptr, 0);
        m->stream_trace = nullptr;
    }
    if (rc == MODEL_OK && cudaMemcpyAsync(out, d, per * kernels * sizeof(unsigned long long), cudaMemcpyDeviceToHost,
                                          m->st) != cudaSuccess)
        rc = MODEL_ERR_DEVICE;
    if (rc == MODEL_OK) rc = finish(m);
    cudaStreamSynchronize(m->st);
    cudaFree(d);
    return rc;
}

model_status model_debug_wait_drill(model* m, uint64_t limit_ns) {
    if (!m || limit_ns == 0) return MODEL_ERR_ARG;
    m->drill_ns = limit_ns;
    return MODEL_OK;
}

model_status model_set_step_kernel(model* m, int kind) {
    if (!m || (kind != TIE_STEP_PERSISTENT && kind != TIE_STEP_CHAINED && kind != TIE_STEP_STREAM))
        return MODEL_ERR_ARG;
    if (kind != m->step_kind) drop_graphs(m);
    m->step_kind = kind;
    return MODEL_OK;
}

model_status model_time_kernel(model* m, int kernel, size_t rows, size_t context, int iters,
                               float* avg_ms) {
    if (!m || !avg_ms || rows == 0 || context == 0 || iters <= 0) return MODEL_ERR_ARG;
    if (!m->pool || (int)rows > m->pool->n_seq || (int)context > m->pool->capacity) return MODEL_ERR_CAPACITY;
    const int E = m->cfg.n_embd, H = m->cfg.n_head, V = m->cfg.vocab_size, B = (int)rows;
    const bool small = B <= kGemvRows;
    cudaStream_t st = m->st;
    model_status rc = ensure_slots(m, rows, m->pool->capacity);
    if (rc != MODEL_OK) return rc;
    if (kernel == TIE_KERNEL_PREFILL_ATTENTION || kernel == TIE_KERNEL_PREFILL_FC)
        if ((rc = ensure_rows(m, rows * context)) != MODEL_OK) return rc;
    // deterministic, finite contents for every operand
    std::vector<int32_t> lens(rows, (int32_t)context - 1), toks(rows, 1);
    if ((rc = set_slot_state(m, rows, toks.data(), lens.data())) != MODEL_OK) return rc;
    if ((rc = map_pages(m, rows, context)) != MODEL_OK) return rc;
    const size_t R = kernel >= TIE_KERNEL_PREFILL_ATTENTION ? rows * context : rows;
    CU(cudaMemsetAsync(m->qkv, 0, R * 3 * E * sizeof(float), st));
    CU(cudaMemsetAsync(m->x, 0, R * E * sizeof(float), st));
    CU(cudaMemsetAsync(m->xb, 0, R * E * sizeof(float), st));
    CU(cudaMemsetAsync(m->ff, 0, R * 4 * E * sizeof(float), st));
    const Layer& w = m->layers[0];
    const PagedKV view = layer_view(m->pool, 0);
    const int splits = attn_decode_max_splits(m->pool->capacity);
    const Mat xb{m->xb, m->xb_hi, m->xb_lo}, ff{m->ff, m->ff_hi, m->ff_lo};
    CU(cudaMemsetAsync(m->xb_hi, 0, R * E * sizeof(float), st));
    CU(cudaMemsetAsync(m->xb_lo, 0, R * E * sizeof(float), st));
    CU(cudaMemsetAsync(m->ff_hi, 0, R * 4 * E * sizeof(float), st));
    CU(cudaMemsetAsync(m->ff_lo, 0, R * 4 * E * sizeof(float), st));
    const bool stream = use_stream(m, B);
    const StreamParams sbase = stream_base(m, B);
    auto once = [&]() -> model_status {
        if (stream && kernel >= TIE_KERNEL_DECODE_ATTENTION && kernel <= TIE_KERNEL_DECODE_HEAD) {
            StreamParams p = sbase;
            switch (kernel) {
                case TIE_KERNEL_DECODE_ATTENTION:
                    CU(launch_attn_chunks(m->qkv, m->d_lens, B, H, view, splits, m->d_part, st));
                    return MODEL_OK;
                case TIE_KERNEL_DECODE_QKV:
                    p.epi = EPI_QKV_KV; p.pro = STREAM_PRO_LN;
                    p.x = m->x; p.ldx = E; p.ln_g = w.ln1_w; p.ln_b = w.ln1_b;
                    stream_weights(p, w.qkv_w, qmat(m, 0, 0), w.qkv_b);
                    p.y = m->qkv; p.ldy = 3 * E; p.N = 3 * E; p.K = E; p.kv = view;
                    break;
                case TIE_KERNEL_DECODE_FC:
                    p.epi = EPI_BIAS_GELU; p.pro = STREAM_PRO_LN;
                    p.x = m->x; p.ldx = E; p.ln_g = w.ln2_w; p.ln_b = w.ln2_b;
                    stream_weights(p, w.fc_w, qmat(m, 0, 2), w.fc_b);
                    p.y = m->ff; p.ldy = 4 * E; p.N = 4 * E; p.K = E;
                    break;
                case TIE_KERNEL_DECODE_MLP_PROJ:
                    p.epi = EPI_BIAS_RESID; p.pro = STREAM_PRO_PLAIN;
                    p.x = m->ff; p.ldx = 4 * E;
                    stream_weights(p, w.mlp_w, qmat(m, 0, 3), w.mlp_b);
                    p.y = m->x; p.ldy = E; p.N = E; p.K = 4 * E;
                    break;
                default: {   // the head
                    const QMat qh = qmat(m, m->cfg.n_layer, 0);
                    p.head = 1; p.pro = STREAM_PRO_LN;
                    p.x = m->x; p.ldx = E; p.ln_g = m->lnf_w; p.ln_b = m->lnf_b;
                    stream_weights(p, m->wte, qh, nullptr);
                    p.y = m->logits; p.ldy = V; p.N = V; p.K = E;
                    p.part_val = m->d_am_val; p.part_idx = m->d_am_idx;
                    CU(launch_stream_gemv(p, st));
                    CU(launch_argmax_finalize(m->d_am_val, m->d_am_idx, stream_head_blocks(V, E, qh.wt, B), B,
                                              m->d_next, st));
                    return MODEL_OK;
                }
            }
            CU(launch_stream_gemv(p, st));
            return MODEL_OK;
        }
        switch (kernel) {
            case TIE_KERNEL_DECODE_ATTENTION:
                CU(launch_attn_decode(m->qkv, m->d_lens, B, H, view, splits, m->d_part, small ? m->attn : nullptr,
                                      nullptr, st, small ? nullptr : m->attn_hi, small ? nullptr : m->attn_lo,
                                      m->d_attn_cnt, m->d_err));
                return MODEL_OK;
            case TIE_KERNEL_DECODE_QKV:
                if (small) {
                    const QMat q = qmat(m, 0, 0);
                    CU(launch_dec_gemv(m->xb, E, nullptr, nullptr, 0.f, w.qkv_w, w.qkv_b, m->qkv,
                                       3 * E, B, 3 * E, E, EPI_QKV_KV, &view, m->d_lens, st, q.wt, q.q, q.s));
                    return MODEL_OK;
                }
                return matmul(m, true, B, xb, E, Mat{w.qkv_w, w.qkv_hi, w.qkv_lo}, 3 * E, E, w.qkv_b, EPI_BIAS,
                              m->qkv, nullptr, nullptr, 3 * E);
            case TIE_KERNEL_DECODE_FC:
                if (small) {
                    const QMat q = qmat(m, 0, 2);
                    CU(launch_dec_gemv(m->xb, E, nullptr, nullptr, 0.f, w.fc_w, w.fc_b, m->ff,
                                       4 * E, B, 4 * E, E, EPI_BIAS_GELU, nullptr, nullptr, st, q.wt, q.q, q.s));
                    return MODEL_OK;
                }
                return matmul(m, true, B, xb, E, Mat{w.fc_w, w.fc_hi, w.fc_lo}, 4 * E, E, w.fc_b, EPI_BIAS_GELU,
                              nullptr, m->ff_hi, m->ff_lo, 4 * E);
            case TIE_KERNEL_DECODE_MLP_PROJ:
                if (small) {
                    const QMat q = qmat(m, 0, 3);
                    CU(launch_dec_gemv(m->ff, 4 * E, nullptr, nullptr, 0.f, w.mlp_w, w.mlp_b, m->x, E, B, E, 4 * E,
                                       EPI_BIAS_RESID, nullptr, nullptr, st, q.wt, q.q, q.s));
                    return MODEL_OK;
                }
                return matmul(m, true, B, ff, 4 * E, Mat{w.mlp_w, w.mlp_hi, w.mlp_lo}, E, 4 * E, w.mlp_b,
                              EPI_BIAS_RESID, m->x, nullptr, nullptr, E);
            case TIE_KERNEL_DECODE_HEAD:
                if (small) {
                    const QMat q = qmat(m, m->cfg.n_layer, 0);
                    CU(launch_dec_head(m->xb, E, nullptr, nullptr, 0.f, m->wte, m->logits, V,
                                       B, V, E, m->d_am_val, m->d_am_idx, st, q.wt, q.q, q.s));
                    CU(launch_argmax_finalize(m->d_am_val, m->d_am_idx, dec_head_blocks(V, E, q.wt, B), B, m->d_next,
                                              st));
                    return MODEL_OK;
                } else {
                    model_status r = matmul(m, true, B, xb, E, Mat{m->wte, m->wte_hi, m->wte_lo}, V, E, nullptr,
                                            EPI_STORE, m->logits, nullptr, nullptr, V);
                    if (r != MODEL_OK) return r;
                    CU(launch_argmax_rows(m->logits, V, B, V, 1, 0, m->d_next, st));
                    return MODEL_OK;
                }
            case TIE_KERNEL_PREFILL_ATTENTION:
                CU(launch_attn_prefill(m->qkv, B, (int)context, H, nullptr, nullptr, st, m->attn_hi, m->attn_lo, m->d_err));
                return MODEL_OK;
            case TIE_KERNEL_PREFILL_FC:
                return matmul(m, false, (int)R, xb, E, Mat{w.fc_w, w.fc_hi, w.fc_lo}, 4 * E, E, w.fc_b,
                              EPI_BIAS_GELU, nullptr, m->ff_hi, m->ff_lo, 4 * E);
            case TIE_KERNEL_DECODE_STEP:
                // the step without advancing: every launch sees the same lengths
                if (!step_applies(m, B, m->pool)) return MODEL_ERR_ARG;
                return run_step(m, B, m->pool, false, nullptr, 0);
        }
        return MODEL_ERR_ARG;
    };
    if ((rc = once()) != MODEL_OK) return rc;  // warm
    cudaEvent_t a, b;
    CU(cudaEventCreate(&a));
    CU(cudaEventCreate(&b));
    CU(cudaEventRecord(a, st));
    for (int i = 0; i < iters; ++i)
        if ((rc = once()) != MODEL_OK) return rc;
    CU(cudaEventRecord(b, st));
    CU(cudaEventSynchronize(b));
    float ms = 0.f;
    CU(cudaEventElapsedTime(&ms, a, b));
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    *avg_ms = ms / (float)iters;
    return MODEL_OK;
}

}  // extern "C"
