// sd_engine.cu -- model context: GGUF parsing, weight upload + repack, KV ring, the S-token forward
// (captured in CUDA graphs with programmatic dependent launch between kernels) and the device-driven
// generation loops, behind the C ABI of include/specdec_b200.h.
//
// Forward of S tokens at positions pos..pos+S-1 (mistral/mistral_model.h:818-899 per token,
// batched like metal_forward_batch, mistral/mistral_infer.m:103-179):
//   embed + RMSNorm + Q8_0            k_norm_quant<0>
//   per layer:
//     QKV matvec + RoPE + KV write    k_gemv<EPI_QKV>      (Wq|Wk|Wv stacked rows)
//     GQA attention + Q8_0            k_attn_partial, k_attn_combine
//     o-proj matvec                   k_gemv<EPI_STORE>    (K-split partials)
//     [TP: all-reduce]
//     residual + RMSNorm + Q8_0       k_norm_quant<1>
//     gate|up matvec + SiLU + Q8_0    k_gemv<EPI_SILU_Q8>  (gate/up row-groups interleaved)
//     down matvec                     k_gemv<EPI_STORE>
//     [TP: all-reduce]
//     residual + next RMSNorm + Q8_0  k_norm_quant<1>
//   LM head                           k_gemv<EPI_STORE>, k_argmax
// Every kernel reads the position and valid-token count from a device control block, so one graph per
// S replays for any position; every kernel is batch invariant, so a token's logits in an S=K+1 verify
// are bit-identical to its S=1 decode logits.
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "sd_attn.h"
#include "sd_fwd.h"
#include "sd_kquant.h"
#include "sd_dev.cuh"
#include "sd_common.cuh"
#include "sd_host.h"
#include "sd_spec.h"
#include "specdec_b200.h"

using namespace sd;

static_assert(sd::kMaxVerify == SD_MAX_VERIFY, "verify width differs between the ABI and the kernels");

namespace {

// ---------------------------------------------------------------------------------------------
// GGUF v3 (the format mistral/gguf_loader.h:148-325 reads)
// ---------------------------------------------------------------------------------------------
struct GTensor {
    std::string name;
    uint32_t type;
    uint64_t ne[4];
    uint32_t nd;
    uint64_t off;  // absolute byte offset in the image
};

struct GGUF {
    const uint8_t* base = nullptr;
    size_t len = 0;
    int dim = 0, hidden = 0, n_layers = 0, n_heads = 0, n_kv = 0, vocab = 0, ctx_len = 0;
    float theta = 10000.f, eps = 1e-5f;
    int bos = 1, eos = 2;
    uint32_t version = 0;
    size_t data_start = 0;
    std::vector<GTensor> t;
    const GTensor* find(const std::string& n) const {
        for (auto& x : t)
            if (x.name == n) return &x;
        return nullptr;
    }
};

struct Rd {
    const uint8_t* b;
    size_t pos, len;
    bool ok = true;
    bool need(size_t n) {
        if (pos + n > len) ok = false;
        return ok;
    }
    uint64_t u(int n) {
        if (!need(n)) return 0;
        uint64_t v = 0;
        memcpy(&v, b + pos, n);
        pos += n;
        return v;
    }
    float f32() {
        uint32_t v = (uint32_t)u(4);
        float f;
        memcpy(&f, &v, 4);
        return f;
    }
    double f64() {
        uint64_t v = u(8);
        double d;
        memcpy(&d, &v, 8);
        return d;
    }
    std::string str() {
        uint64_t n = u(8);
        if (!need(n)) return std::string();
        std::string s((const char*)b + pos, n);
        pos += n;
        return s;
    }
};

enum { GV_U8 = 0, GV_I8, GV_U16, GV_I16, GV_U32, GV_I32, GV_F32, GV_BOOL, GV_STR, GV_ARR, GV_U64, GV_I64, GV_F64 };

int gv_size(uint32_t t) {
    switch (t) {
        case GV_U8: case GV_I8: case GV_BOOL: return 1;
        case GV_U16: case GV_I16: return 2;
        case GV_U32: case GV_I32: case GV_F32: return 4;
        case GV_U64: case GV_I64: case GV_F64: return 8;
    }
    return -1;
}

double gv_num(Rd& r, uint32_t t) {
    switch (t) {
        case GV_U8: case GV_BOOL: return (double)(uint8_t)r.u(1);
        case GV_I8: return (double)(int8_t)r.u(1);
        case GV_U16: return (double)(uint16_t)r.u(2);
        case GV_I16: return (double)(int16_t)r.u(2);
        case GV_U32: return (double)(uint32_t)r.u(4);
        case GV_I32: return (double)(int32_t)r.u(4);
        case GV_U64: return (double)r.u(8);
        case GV_I64: return (double)(int64_t)r.u(8);
        case GV_F32: return (double)r.f32();
        case GV_F64: return r.f64();
    }
    r.ok = false;
    return 0;
}

void gv_skip(Rd& r, uint32_t t, int depth = 0) {
    if (depth > 4) { r.ok = false; return; }
    if (t == GV_STR) { r.str(); return; }
    if (t == GV_ARR) {
        uint32_t at = (uint32_t)r.u(4);
        uint64_t n = r.u(8);
        int sz = gv_size(at);
        if (sz > 0) {
            if (r.need(n * sz)) r.pos += n * sz;
            return;
        }
        for (uint64_t i = 0; i < n && r.ok; ++i) gv_skip(r, at, depth + 1);
        return;
    }
    int sz = gv_size(t);
    if (sz < 0) { r.ok = false; return; }
    if (r.need(sz)) r.pos += sz;
}

bool key_is(const std::string& k, const char* suffix) {
    return k == std::string("llama.") + suffix || k == std::string("mistral.") + suffix;
}

int gguf_parse(const void* base, size_t len, GGUF& g) {
    Rd r{(const uint8_t*)base, 0, len};
    g.base = (const uint8_t*)base;
    g.len = len;
    if (r.u(4) != 0x46554747u) return fail(SD_ERR_FORMAT, "not a GGUF file");
    uint32_t ver = (uint32_t)r.u(4);
    if (ver < 2) return fail(SD_ERR_FORMAT, "GGUF version %u unsupported", ver);
    g.version = ver;
    uint64_t n_t = r.u(8), n_kv = r.u(8);
    if (!r.ok || n_t > 100000 || n_kv > 100000) return fail(SD_ERR_FORMAT, "GGUF header truncated");
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        std::string k = r.str();
        uint32_t vt = (uint32_t)r.u(4);
        if (key_is(k, "embedding_length")) g.dim = (int)gv_num(r, vt);
        else if (key_is(k, "feed_forward_length")) g.hidden = (int)gv_num(r, vt);
        else if (key_is(k, "block_count")) g.n_layers = (int)gv_num(r, vt);
        else if (key_is(k, "attention.head_count")) g.n_heads = (int)gv_num(r, vt);
        else if (key_is(k, "attention.head_count_kv")) g.n_kv = (int)gv_num(r, vt);
        else if (key_is(k, "context_length")) g.ctx_len = (int)gv_num(r, vt);
        else if (key_is(k, "rope.freq_base")) g.theta = (float)gv_num(r, vt);
        else if (key_is(k, "attention.layer_norm_rms_epsilon")) g.eps = (float)gv_num(r, vt);
        else if (k == "tokenizer.ggml.bos_token_id") g.bos = (int)gv_num(r, vt);
        else if (k == "tokenizer.ggml.eos_token_id") g.eos = (int)gv_num(r, vt);
        else if (k == "tokenizer.ggml.tokens" && vt == GV_ARR) {
            size_t save = r.pos;
            uint32_t at = (uint32_t)r.u(4);
            uint64_t n = r.u(8);
            (void)at;
            g.vocab = (int)n;
            r.pos = save;
            gv_skip(r, vt);
        } else gv_skip(r, vt);
    }
    for (uint64_t i = 0; i < n_t && r.ok; ++i) {
        GTensor t;
        t.name = r.str();
        t.nd = (uint32_t)r.u(4);
        if (t.nd > 4) return fail(SD_ERR_FORMAT, "tensor %s: %u dims", t.name.c_str(), t.nd);
        for (int d = 0; d < 4; ++d) t.ne[d] = 1;
        for (uint32_t d = 0; d < t.nd; ++d) t.ne[d] = r.u(8);
        t.type = (uint32_t)r.u(4);
        t.off = r.u(8);
        g.t.push_back(t);
    }
    if (!r.ok) return fail(SD_ERR_FORMAT, "GGUF metadata truncated");
    const size_t data_start = (r.pos + 31) / 32 * 32;   // gguf_loader.h:280-281
    g.data_start = data_start;
    for (auto& t : g.t) {
        t.off += data_start;
        uint64_t nel = t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3];
        uint64_t bytes = t.type == 2 ? nel / 32 * 18 : t.type == 0 ? nel * 4 : t.type == 1 ? nel * 2
                       : t.type == 12 ? nel / 256 * 144 : t.type == 14 ? nel / 256 * 210 : 0;
        if (bytes == 0 || t.off + bytes > len) return fail(SD_ERR_FORMAT, "tensor %s out of range", t.name.c_str());
    }
    if (g.dim <= 0 || g.n_layers <= 0 || g.n_heads <= 0 || g.n_kv <= 0 || g.hidden <= 0)
        return fail(SD_ERR_FORMAT, "GGUF lacks model hyper-parameters");
    if (g.vocab <= 0) {
        const GTensor* e = g.find("token_embd.weight");
        if (e) g.vocab = (int)e->ne[1];
    }
    return SD_OK;
}

struct LayerW {
    uint8_t *qkv = nullptr, *wo = nullptr, *w13 = nullptr, *w2 = nullptr;
    float *rms_att = nullptr, *rms_ffn = nullptr;
};

struct Plan {  // a matvec launch configuration
    GemvArgs a;
    int grid = 0;
    size_t smem = 0;
};

}  // namespace

struct sd_ctx {
    int dev = 0;
    cudaStream_t st = nullptr;
    bool use_graphs = true, use_pdl = true;
    bool prefill_gemm = true;       // long prompts through the batched engine's GEMMs (gemm_prefill)
    bool pf_unsupported = false;    // the batched engine declined this model: matvec prefill only
    sd_batch* pf = nullptr;         // the prefill batch over this context's ring, made at the first long prompt
    // model
    int dim, hidden, n_layers, n_heads, n_kv, hd, vocab, max_seq, bos, eos;
    float theta, eps;
    int tp_rank = 0, tp_size = 1;
    int nh_l, nkv_l, q_rows, kv_rows, hid_l, qkv_rows;
    int MB;  // max tokens per forward
    std::vector<LayerW> L;
    uint8_t* embd = nullptr;
    uint8_t* lm = nullptr;
    int embd_type = 2;         // token_embd.weight: Q4_0 (2) or Q4_K (12), rows as in the GGUF
    int lm_type = 2;           // output.weight: Q4_0 (2, tile layout) or Q6_K (14) / Q4_K (12) (sd_kquant.h layout)
    float* xn = nullptr;       // [MB][dim] final-norm output for a K-quant LM head
    float *rms_final = nullptr, *theta_inv = nullptr;
    __half *kc = nullptr, *vc = nullptr;      // [n_layers][max_seq][kv_rows]
    __half *dkc = nullptr, *dvc = nullptr;    // self-spec drafter KV [draft_layers][max_seq][kv_rows]
    int draft_layers_alloc = 0;
    int draft_kv_hist = 0, draft_kv_layers = 0;  // drafter K/V prefilled for history[0 .. draft_kv_hist) at this depth
    size_t weight_bytes = 0, kv_bytes = 0;
    // buffers
    float* x = nullptr;        // [MB][dim]
    float* y = nullptr;        // [ypart][MB][dim]
    int ypart_max = 8;
    Q8Planes act{}, hact{};
    float* q = nullptr;        // [MB][q_rows]
    float2* part_ml = nullptr;
    float* part_acc = nullptr;
    int attn_chunk = 64, max_chunks = 0;
    float* logits = nullptr;   // [kMaxVerify][vocab]
    float* probs = nullptr;    // [vocab]
    int* argmax = nullptr;     // [kMaxVerify]
    DevCtrl* ctrl_sub = nullptr;  // [kMaxVerify] control blocks of the forwards a wide verify batch splits into
    DevCtrl* ctrl = nullptr;   // verify / decode forward
    DevCtrl* dctrl = nullptr;  // self-spec drafter chain
    int* err = nullptr;
    // generation
    GenState* gs = nullptr;
    GenState* gs_h = nullptr;
    int* g_out = nullptr;
    int* g_hist = nullptr;
    int g_cap = 0;
    // graphs
    cudaGraphExec_t fwd_graph[kMaxVerify + 1] = {};
    cudaGraphExec_t fwd_graph_kv[kMaxVerify + 1] = {};  // prefill forwards: K/V only, no LM head
    cudaGraphExec_t iter_graph = nullptr;
    int iter_key[6] = {-1, -1, -1, -1, -1, -1};
    GenParamsDev iter_p{};
    unsigned long long rng_start = 1ull << 20;  // Philox counter the next decode loop starts from
    // persistent forward kernel (forward_kernel = 1)
    bool fused = false;
    FwdLayer* d_layers = nullptr;  // device copy of the per-layer weight pointers
    float* ssq = nullptr;          // [MB][dim/16] group sums of squares of x
    void* img_mem = nullptr;       // activation images (norm input, head outputs, SiLU output)
    ActImage img_un{}, img_attn{}, img_h{};
    unsigned* fsync = nullptr;     // grid barrier + slice counters
    MvPhase ph_qkv{}, ph_wo{}, ph_w13{}, ph_w2{}, ph_lm{};
    int fwd_stages = 0, fwd_grid = 0;
    size_t fwd_smem = 0;
    // TP
    void* nccl = nullptr;
    void* tp_mem = nullptr;                 // exchange region: [2][tp_buf] floats + kMaxTp flags
    size_t tp_buf = 0;                      // floats per partial-output buffer
    unsigned long long* tp_base = nullptr;  // reductions completed before the current forward
    TpXchg tpx{};                           // peers connected: the norm kernels do the all-reduce
    std::vector<void*> tp_opened;           // peer regions opened through CUDA IPC
};

namespace {

int ck(cudaError_t e, const char* what) { return e == cudaSuccess ? SD_OK : cuda_fail(e, what); }

#define CK(expr, what)                                   \
    do {                                                 \
        int _rc = ck((expr), (what));                    \
        if (_rc) return _rc;                             \
    } while (0)

template <class T>
int dalloc(T** p, size_t n, size_t* acc = nullptr) {
    cudaError_t e = cudaMalloc((void**)p, n * sizeof(T));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
    if (acc) *acc += n * sizeof(T);
    return SD_OK;
}

// Upload AoS rows [r0, r0+rows) x column blocks [cb0, cb0 + cols/32) of a GGUF Q4_0 tensor and repack
// them into dst at the rows given by map.
int upload_q4(sd_ctx* c, const GGUF& g, const GTensor* t, int r0, int rows, int cb0, int cols, RowMap map,
              uint8_t* dst, uint8_t* staging, size_t staging_bytes) {
    if (!t || t->type != 2) return fail(SD_ERR_FORMAT, "tensor %s missing or not Q4_0", t ? t->name.c_str() : "?");
    const size_t row_bytes = (size_t)t->ne[0] / 32 * 18;
    const uint8_t* src = g.base + t->off + (size_t)r0 * row_bytes;
    // contiguous rows (whole width) are uploaded once; column slices upload the needed row span
    const size_t span = (size_t)rows * row_bytes;
    if (span > staging_bytes) return fail(SD_ERR_INVALID, "staging buffer too small");
    CK(cudaMemcpyAsync(staging, src, span, cudaMemcpyHostToDevice, c->st), "weight upload");
    CK(launch_repack(staging + (size_t)cb0 * 18, rows, cols, row_bytes, map, dst, c->st), "repack");
    CK(cudaStreamSynchronize(c->st), "repack");
    return SD_OK;
}

int upload_f32(sd_ctx* c, const GGUF& g, const char* name, float** out, int n) {
    const GTensor* t = g.find(name);
    if (!t || t->type != 0 || (int)(t->ne[0] * t->ne[1]) != n) return fail(SD_ERR_FORMAT, "tensor %s missing or not F32[%d]", name, n);
    int rc = dalloc(out, n, &c->weight_bytes);
    if (rc) return rc;
    CK(cudaMemcpy(*out, g.base + t->off, (size_t)n * 4, cudaMemcpyHostToDevice), "upload");
    return SD_OK;
}

int build_plan(sd_ctx* c, Plan& p, int epi, const uint8_t* w, int rows, int K, int rg_per_unit, int S, int kparts) {
    GemvArgs& a = p.a;
    a = GemvArgs{};
    a.w = w;
    a.n_rg = qmat_row_groups(rows);
    a.nq = K / 128;
    a.K = K;
    a.rg_per_unit = rg_per_unit;
    a.n_units = a.n_rg / rg_per_unit;
    a.S = S;
    a.kparts = kparts;
    a.out_rows = rows;
    a.err = c->err;
    return gemv_plan(a, c->dev, &p.grid, &p.smem);
}

// K split of a matvec, fixed for every S: the split the planner picks at the largest S.  A split that
// changed with S would change the summation order, and a token's result must not depend on how many
// tokens share its forward (verify rows equal single-token decode rows bit for bit).
int fixed_kparts(sd_ctx* c, int rows, int K, int* kparts) {
    Plan p;
    int rc = build_plan(c, p, EPI_STORE, nullptr, rows, K, kRPW, kMaxS, 0);
    if (rc) return rc;
    *kparts = p.a.kparts;
    return SD_OK;
}

int launch_plan(sd_ctx* c, int epi, Plan& p) {
    cudaError_t e = launch_gemv(epi, p.a, p.grid, p.smem, c->st, c->use_pdl);
    return e == cudaSuccess ? SD_OK : cuda_fail(e, "matvec launch");
}

// Plan of one matvec phase of the persistent forward (the same K split and chunk as the per-op
// path); false if the shape does not fit the kernel's activation buffer.
bool fwd_phase(MvPhase& p, int rows, int K, int rpu, int kparts) {
    const int n_rg = qmat_row_groups(rows);
    if (n_rg % rpu || K % 128 || kparts < 1) return false;
    p.n_units = n_rg / rpu;
    p.rpu = rpu;
    p.nq = K / 128;
    p.kparts = kparts;
    if (p.nq % kparts) return false;
    const int nqp = p.nq / kparts;
    p.chunk = gemv_chunk(nqp);
    return nqp % p.chunk == 0 && nqp <= 32;
}

// Set up the persistent forward kernel; leaves c->fused false (per-op kernels) where it does not apply.
int setup_fused(sd_ctx* c) {
    int coop = 0;
    CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, c->dev), "device attribute");
    if (!coop) return SD_OK;
    int kp_o = 0, kp_d = 0, rc;
    if ((rc = fixed_kparts(c, c->dim, c->q_rows, &kp_o)) || (rc = fixed_kparts(c, c->dim, c->hid_l, &kp_d))) return rc;
    if (kp_o > c->ypart_max || kp_d > c->ypart_max) return SD_OK;
    if (!fwd_phase(c->ph_qkv, c->qkv_rows, c->dim, kRPW, 1) || !fwd_phase(c->ph_wo, c->dim, c->q_rows, kRPW, kp_o) ||
        !fwd_phase(c->ph_w13, 2 * c->hid_l, c->dim, 2 * kRPW, 1) || !fwd_phase(c->ph_w2, c->dim, c->hid_l, kRPW, kp_d) ||
        !fwd_phase(c->ph_lm, c->vocab, c->dim, kRPW, 1))
        return SD_OK;
    const int max_smem = device_max_smem(c->dev);
    c->fwd_stages = fwd_pick_stages(max_smem);
    if (c->fwd_stages < 3) return SD_OK;
    c->fwd_smem = fwd_smem_bytes(c->fwd_stages);
    CK(fwd_init_attrs(max_smem), "cudaFuncSetAttribute (forward)");
    int per_sm = 0;
    CK(fwd_blocks_per_sm(c->fwd_smem, &per_sm), "occupancy");
    if (per_sm < 1) return SD_OK;
    c->fwd_grid = device_sm_count(c->dev);
    std::vector<FwdLayer> hl(c->n_layers);
    for (int l = 0; l < c->n_layers; ++l)
        hl[l] = FwdLayer{c->L[l].qkv, c->L[l].wo, c->L[l].w13, c->L[l].w2, c->L[l].rms_att, c->L[l].rms_ffn};
    if ((rc = dalloc(&c->d_layers, hl.size())) || (rc = dalloc(&c->ssq, (size_t)c->MB * (c->dim / 16))) ||
        (rc = dalloc(&c->fsync, fwd_sync_words(c->dim))))
        return rc;
    {
        const size_t bu = act_image_bytes(c->dim / 32), ba = act_image_bytes(c->q_rows / 32),
                     bh = act_image_bytes(c->hid_l / 32);
        uint8_t* p = nullptr;
        if ((rc = dalloc(&p, bu + ba + bh))) return rc;
        CK(cudaMemset(p, 0, bu + ba + bh), "memset");
        c->img_mem = p;
        c->img_un = act_image_at(p, c->dim / 32);
        c->img_attn = act_image_at(p + bu, c->q_rows / 32);
        c->img_h = act_image_at(p + bu + ba, c->hid_l / 32);
    }
    CK(cudaMemcpy(c->d_layers, hl.data(), hl.size() * sizeof(FwdLayer), cudaMemcpyHostToDevice), "layer table");
    CK(cudaMemset(c->fsync, 0, fwd_sync_words(c->dim) * sizeof(unsigned)), "memset");
    c->fused = true;
    return SD_OK;
}

// A K-quant LM head (Q6_K / Q4_K output.weight) on the final residual c->x: the final RMSNorm in fp32, the
// fp32-activation K-quant matvec and the argmax (mistral/mistral_model.h:1110-1122 non-Q4_0 branch).  Both forward
// paths end with the same x, so their logits agree bit for bit.
int enqueue_kq_head(sd_ctx* c, int S, DevCtrl* ctrl, int row0) {
    CK(launch_final_norm(c->x, c->rms_final, c->xn, c->dim, c->eps, S, ctrl, c->st), "final norm");
    CK(launch_kq_matvec(c->lm_type, c->lm, c->vocab, c->dim, c->xn, c->logits + (size_t)row0 * c->vocab, c->vocab, S, ctrl,
                        c->st), "K-quant LM head");
    CK(launch_argmax(c->logits + (size_t)row0 * c->vocab, c->vocab, S, c->argmax + row0, ctrl, c->st, false), "argmax");
    return SD_OK;
}

// One forward as a single persistent kernel (then the argmax kernel when logits are wanted).
int enqueue_forward_fused(sd_ctx* c, int S, int n_layers, __half* k, __half* v, DevCtrl* ctrl, bool logits_and_argmax,
                          int row0) {
    FwdArgs a{};
    a.layers = c->d_layers;
    a.n_layers = n_layers;
    a.embd = c->embd;
    a.embd_type = c->embd_type;
    a.rms_out = c->rms_final;
    a.lm = logits_and_argmax && c->lm_type == 2 ? c->lm : nullptr;  // a K-quant head runs after the kernel
    a.dim = c->dim;
    a.hidden = c->hid_l;
    a.q_rows = c->q_rows;
    a.kv_rows = c->kv_rows;
    a.vocab = c->vocab;
    a.head_dim = c->hd;
    a.n_heads = c->nh_l;
    a.n_kvh = c->nkv_l;
    a.S = S;
    a.max_seq = c->max_seq;
    a.eps = c->eps;
    a.q_scale = 1.0f / sqrtf((float)c->hd);
    a.theta_inv = c->theta_inv;
    a.k_cache = k;
    a.v_cache = v;
    a.kv_layer = (size_t)c->max_seq * c->kv_rows;
    a.qkv = c->ph_qkv;
    a.wo = c->ph_wo;
    a.w13 = c->ph_w13;
    a.w2 = c->ph_w2;
    a.lmp = c->ph_lm;
    a.nstage = c->fwd_stages;
    a.x = c->x;
    a.ssq = c->ssq;
    a.un_img = c->img_un;
    a.attn_img = c->img_attn;
    a.h_img = c->img_h;
    a.q = c->q;
    a.attn = c->act;
    a.h = c->hact;
    a.yparts = c->y;
    a.ypart_stride = (size_t)c->MB * c->dim;
    a.sync = c->fsync;
    a.part_ml = c->part_ml;
    a.part_acc = c->part_acc;
    a.attn_chunk = c->attn_chunk;
    a.max_chunks = c->max_chunks;
    a.logits = c->logits + (size_t)row0 * c->vocab;
    a.tokens = nullptr;
    a.ctrl = ctrl;
    a.err = c->err;
    a.tp = c->tpx;
    CK(cudaMemsetAsync(c->fsync, 0, fwd_sync_words(c->dim) * sizeof(unsigned), c->st), "memset");
    CK(launch_forward(a, c->fwd_grid, c->fwd_smem, c->st), "forward launch");
    if (c->tpx.n > 1) CK(launch_tp_advance(c->tp_base, 2 * n_layers, c->st), "tp advance");
    if (!logits_and_argmax) return SD_OK;
    if (c->lm_type != 2) return enqueue_kq_head(c, S, ctrl, row0);
    // the LM head phase reduced the argmax keys (first index on ties) into the sync words
    CK(launch_argmax_keys(reinterpret_cast<const unsigned long long*>(c->fsync + 32), S, c->argmax + row0, ctrl, c->st),
       "argmax");
    return SD_OK;
}

// Output buffer of reduction idx (0-based within a forward) of this rank's o-proj / down-proj: with
// peers connected, the exchange buffer of the reduction's parity (sequence numbers start at an even base
// and grow by 2 * n_layers per forward), else the local partial-output buffer.
float* tp_out(sd_ctx* c, int idx) {
    if (c->tpx.n > 1) return c->tpx.y[c->tp_rank] + (size_t)((idx + 1) & 1) * c->tp_buf;
    return c->y;
}

TpXchg tp_args(sd_ctx* c, int idx) {
    TpXchg t = c->tpx;
    t.idx = idx;
    return t;
}

// Tensor parallelism: this rank's o-proj / down-proj output is a partial sum over its input columns.
// Add its K slices into slice 0, then sum slice 0 over the ranks; the norm then adds one slice.
int tp_reduce(sd_ctx* c, int S, int* yparts) {
    if (c->tp_size <= 1 || c->tpx.n > 1) return SD_OK;  // peer path: the next norm kernel reduces
    const size_t n = (size_t)S * c->dim;
    if (*yparts > 1) CK(launch_sum_parts(c->y, c->y, (int)n, *yparts, (size_t)c->MB * c->dim, c->st), "sum parts");
    *yparts = 1;
    return nccl_allreduce_sum(c->nccl, c->y, n, c->st);
}

// One decode layer l of S tokens in the kernel-per-op path (mistral/mistral_model.h:818-899): the Q8_0 input of
// the attention norm is in c->act; ends with x updated and the Q8_0 of the next norm (weight w_next) in c->act.
int enqueue_layer_perop(sd_ctx* c, int l, int S, __half* k, __half* v, DevCtrl* ctrl, NormArgs& na, const float* w_next) {
    const bool pdl = c->use_pdl;
    const size_t kv_layer = (size_t)c->max_seq * c->kv_rows;
    LayerW& W = c->L[l];
    // QKV + RoPE + KV write
    Plan pq;
    int rc = build_plan(c, pq, EPI_QKV, W.qkv, c->qkv_rows, c->dim, kRPW, S, 1);
    if (rc) return rc;
    pq.a.act = c->act;
    pq.a.ctrl = ctrl;
    pq.a.q_out = c->q;
    pq.a.k_cache = k + l * kv_layer;
    pq.a.v_cache = v + l * kv_layer;
    pq.a.q_rows = c->q_rows;
    pq.a.kv_rows = c->kv_rows;
    pq.a.max_seq = c->max_seq;
    pq.a.head_dim = c->hd;
    pq.a.theta_inv = c->theta_inv;
    pq.a.q_scale = 1.0f / sqrtf((float)c->hd);
    if ((rc = launch_plan(c, EPI_QKV, pq))) return rc;
    // attention
    AttnArgs aa{};
    aa.q = c->q;
    aa.q_ld = c->q_rows;
    aa.k = k + l * kv_layer;
    aa.v = v + l * kv_layer;
    aa.kv_ld = c->kv_rows;
    aa.n_heads = c->nh_l;
    aa.n_kvh = c->nkv_l;
    aa.S = S;
    aa.max_seq = c->max_seq;
    aa.chunk = c->attn_chunk;
    aa.max_chunks = c->max_chunks;
    aa.part_ml = c->part_ml;
    aa.part_acc = c->part_acc;
    aa.out = c->act;
    aa.ctrl = ctrl;
    CK(launch_attention(aa, 4 * device_sm_count(c->dev), c->st, pdl), "attention");
    // o-proj (K-split partials summed by the next norm)
    Plan po;
    int kp_o = 0, kp_d = 0;
    if ((rc = fixed_kparts(c, c->dim, c->q_rows, &kp_o))) return rc;
    if ((rc = fixed_kparts(c, c->dim, c->hid_l, &kp_d))) return rc;
    if ((rc = build_plan(c, po, EPI_STORE, W.wo, c->dim, c->q_rows, kRPW, S, kp_o))) return rc;
    po.a.act = c->act;
    po.a.ctrl = ctrl;
    po.a.out = tp_out(c, 2 * l);
    po.a.out_ld = c->dim;
    po.a.part_stride = (size_t)c->MB * c->dim;
    if (po.a.kparts > c->ypart_max) return fail(SD_ERR_INVALID, "o-proj K split %d too wide", po.a.kparts);
    if ((rc = launch_plan(c, EPI_STORE, po))) return rc;
    na.w = W.rms_ffn;
    na.yparts = po.a.kparts;
    if ((rc = tp_reduce(c, S, &na.yparts))) return rc;
    na.tp = tp_args(c, 2 * l);
    CK(launch_norm_quant(1, na, c->st, pdl), "norm");
    // gate/up + SiLU + Q8_0
    Plan pg;
    if ((rc = build_plan(c, pg, EPI_SILU_Q8, W.w13, 2 * c->hid_l, c->dim, 4, S, 1))) return rc;
    pg.a.act = c->act;
    pg.a.ctrl = ctrl;
    pg.a.h = c->hact;
    pg.a.hidden = c->hid_l;
    if ((rc = launch_plan(c, EPI_SILU_Q8, pg))) return rc;
    // down
    Plan pd;
    if ((rc = build_plan(c, pd, EPI_STORE, W.w2, c->dim, c->hid_l, kRPW, S, kp_d))) return rc;
    pd.a.act = c->hact;
    pd.a.ctrl = ctrl;
    pd.a.out = tp_out(c, 2 * l + 1);
    pd.a.out_ld = c->dim;
    pd.a.part_stride = (size_t)c->MB * c->dim;
    if (pd.a.kparts > c->ypart_max) return fail(SD_ERR_INVALID, "down K split %d too wide", pd.a.kparts);
    if ((rc = launch_plan(c, EPI_STORE, pd))) return rc;
    na.w = w_next;
    na.yparts = pd.a.kparts;
    if ((rc = tp_reduce(c, S, &na.yparts))) return rc;
    na.tp = tp_args(c, 2 * l + 1);
    CK(launch_norm_quant(1, na, c->st, pdl), "norm");
    return SD_OK;
}

// LM head of the Q8_0 final-norm output in c->act -> logits rows row0.. (and their argmax).
int enqueue_head_perop(sd_ctx* c, int S, DevCtrl* ctrl, int row0) {
    if (c->lm_type != 2) return enqueue_kq_head(c, S, ctrl, row0);
    Plan pl;
    int rc = build_plan(c, pl, EPI_STORE, c->lm, c->vocab, c->dim, kRPW, S, 1);
    if (rc) return rc;
    pl.a.act = c->act;
    pl.a.ctrl = ctrl;
    pl.a.out = c->logits + (size_t)row0 * c->vocab;
    pl.a.out_ld = c->vocab;
    if ((rc = launch_plan(c, EPI_STORE, pl))) return rc;
    CK(launch_argmax(c->logits + (size_t)row0 * c->vocab, c->vocab, S, c->argmax + row0, ctrl, c->st, c->use_pdl),
       "argmax");
    return SD_OK;
}

NormArgs norm_args(sd_ctx* c, int S, DevCtrl* ctrl) {
    NormArgs na{};
    na.x = c->x;
    na.y = c->y;
    na.embd = c->embd;
    na.embd_type = c->embd_type;
    na.out = c->act;
    na.dim = c->dim;
    na.S = S;
    na.eps = c->eps;
    na.ctrl = ctrl;
    na.w = c->L[0].rms_att;
    na.yparts = 1;
    na.ystride = (size_t)c->MB * c->dim;
    na.err = c->err;
    return na;
}

// One forward of S <= MB (template) tokens over n_layers layers on kv ring (k, v); ctrl gives the position,
// the tokens and how many of the S are valid.  Logits / argmax go to rows row0.. of c->logits / c->argmax.
int enqueue_forward_one(sd_ctx* c, int S, int n_layers, __half* k, __half* v, DevCtrl* ctrl, bool logits_and_argmax,
                        int row0) {
    // tensor parallel contexts use the persistent kernel once their peers are connected
    if (c->fused && (c->tp_size == 1 || c->tpx.n > 1))
        return enqueue_forward_fused(c, S, n_layers, k, v, ctrl, logits_and_argmax, row0);
    NormArgs na = norm_args(c, S, ctrl);
    // a slice's control block was just written by the previous kernel: launch after it in full order
    CK(launch_norm_quant(0, na, c->st, c->use_pdl && row0 == 0), "embed");
    for (int l = 0; l < n_layers; ++l) {
        const float* w_next = (l + 1 < n_layers) ? c->L[l + 1].rms_att : c->rms_final;
        int rc = enqueue_layer_perop(c, l, S, k, v, ctrl, na, w_next);
        if (rc) return rc;
    }
    if (c->tpx.n > 1) CK(launch_tp_advance(c->tp_base, 2 * n_layers, c->st), "tp advance");
    if (!logits_and_argmax) return SD_OK;
    return enqueue_head_perop(c, S, ctrl, row0);
}

// Enqueue the forward of S <= kMaxVerify tokens.  A batch wider than MB runs as consecutive forwards of
// MB tokens, each attending to the K/V the previous ones wrote; every reduction is batch invariant, so
// the logits equal those of one wide forward bit for bit.
int enqueue_forward(sd_ctx* c, int S, int n_layers, __half* k, __half* v, DevCtrl* ctrl, bool logits_and_argmax) {
    if (S <= c->MB) return enqueue_forward_one(c, S, n_layers, k, v, ctrl, logits_and_argmax, 0);
    for (int off = 0; off < S; off += c->MB) {
        DevCtrl* cj = ctrl;
        if (off > 0) {
            cj = c->ctrl_sub + off / c->MB;
            CK(launch_ctrl_slice(ctrl, cj, off, c->st), "ctrl slice");
        }
        int rc = enqueue_forward_one(c, std::min(c->MB, S - off), n_layers, k, v, cj, logits_and_argmax, off);
        if (rc) return rc;
    }
    return SD_OK;
}

// Forward graph for S tokens (full depth, target KV, ctrl), built on first use; logits = false leaves out
// the LM head and argmax (prefill chunks whose logits nobody reads).
int forward_graph(sd_ctx* c, int S, bool logits, cudaGraphExec_t* out) {
    cudaGraphExec_t& slot = logits ? c->fwd_graph[S] : c->fwd_graph_kv[S];
    if (slot) {
        *out = slot;
        return SD_OK;
    }
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(c->st, cudaStreamCaptureModeThreadLocal), "capture");
    int rc = enqueue_forward(c, S, c->n_layers, c->kc, c->vc, c->ctrl, logits);
    cudaError_t e = cudaStreamEndCapture(c->st, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return cuda_fail(e, "end capture");
    e = cudaGraphInstantiate(&slot, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(e, "graph instantiate");
    *out = slot;
    return SD_OK;
}

int run_forward(sd_ctx* c, int S, bool logits = true) {
    if (c->use_graphs) {
        cudaGraphExec_t ge;
        int rc = forward_graph(c, S, logits, &ge);
        if (rc) return rc;
        CK(cudaGraphLaunch(ge, c->st), "graph launch");
        return SD_OK;
    }
    return enqueue_forward(c, S, c->n_layers, c->kc, c->vc, c->ctrl, logits);
}

int set_ctrl(sd_ctx* c, DevCtrl* dst, const int32_t* tokens, int S, int pos, bool host_tokens) {
    DevCtrl h{};
    h.pos = pos;
    h.n_valid = S;
    h.done = 0;
    if (host_tokens)
        for (int i = 0; i < S; ++i) h.tokens[i] = tokens[i];
    // the block travels as a kernel argument (copied at launch), so back-to-back stream-ordered calls
    // never share a host staging buffer
    CK(launch_set_ctrl(dst, h, host_tokens ? nullptr : tokens, S, c->st), "ctrl upload");
    return SD_OK;
}

int check_tokens(sd_ctx* c, const int32_t* t, int n) {
    for (int i = 0; i < n; ++i)
        if (t[i] < 0 || t[i] >= c->vocab) return fail(SD_ERR_INVALID, "token %d out of range [0, %d)", t[i], c->vocab);
    return SD_OK;
}

int finish(sd_ctx* c) {
    CK(cudaStreamSynchronize(c->st), "stream sync");
    return check_device_error(c->err, c->st);
}

}  // namespace

// =============================================================================================
extern "C" {

void sd_ctx_opts_default(sd_ctx_opts* o) {
    if (!o) return;
    memset(o, 0, sizeof(*o));
    o->device = 0;
    o->max_seq = 0;
    o->max_batch = 0;
    o->tp_rank = 0;
    o->tp_size = 1;
    o->use_graphs = 1;
    o->use_pdl = 1;
    o->forward_kernel = 1;
    o->prefill_gemm = 1;
}

void sd_ctx_free(sd_ctx* c) {
    if (!c) return;
    cudaSetDevice(c->dev);
    if (c->st) cudaStreamSynchronize(c->st);
    sd_batch_free(c->pf);  // reads this context's weights and ring
    for (auto& g : c->fwd_graph)
        if (g) cudaGraphExecDestroy(g);
    for (auto& g : c->fwd_graph_kv)
        if (g) cudaGraphExecDestroy(g);
    if (c->iter_graph) cudaGraphExecDestroy(c->iter_graph);
    for (auto& W : c->L) {
        cudaFree(W.qkv); cudaFree(W.wo); cudaFree(W.w13); cudaFree(W.w2); cudaFree(W.rms_att); cudaFree(W.rms_ffn);
    }
    cudaFree(c->embd); cudaFree(c->lm); cudaFree(c->xn); cudaFree(c->rms_final); cudaFree(c->theta_inv);
    cudaFree(c->kc); cudaFree(c->vc); cudaFree(c->dkc); cudaFree(c->dvc);
    cudaFree(c->x); cudaFree(c->y); cudaFree(c->act.qs); cudaFree(c->act.d); cudaFree(c->act.sum);
    cudaFree(c->hact.qs); cudaFree(c->hact.d); cudaFree(c->hact.sum); cudaFree(c->q);
    cudaFree(c->part_ml); cudaFree(c->part_acc); cudaFree(c->logits); cudaFree(c->probs); cudaFree(c->argmax);
    cudaFree(c->ctrl); cudaFree(c->dctrl); cudaFree(c->ctrl_sub); cudaFree(c->err); cudaFree(c->gs); cudaFree(c->g_out); cudaFree(c->g_hist);
    cudaFree(c->d_layers); cudaFree(c->ssq); cudaFree(c->fsync);
    cudaFree(c->img_mem);
    for (void* p : c->tp_opened) cudaIpcCloseMemHandle(p);
    cudaFree(c->tp_mem);
    cudaFree(c->tp_base);
    if (c->gs_h) cudaFreeHost(c->gs_h);
    if (c->st) cudaStreamDestroy(c->st);
    delete c;
}

static int ctx_build(const void* base, size_t len, const sd_ctx_opts* opts, sd_ctx** out) {
    clear_error();
    if (!base || !out) return fail(SD_ERR_INVALID, "null argument");
    *out = nullptr;
    if (sd_device_count() == 0) return fail(SD_ERR_NO_DEVICE, "no CUDA device");
    sd_ctx_opts o;
    sd_ctx_opts_default(&o);
    if (opts) o = *opts;
    GGUF g;
    int rc = gguf_parse(base, len, g);
    if (rc) return rc;
    sd_ctx* c = new sd_ctx();
    c->dev = o.device;
    c->use_graphs = o.use_graphs != 0;
    c->use_pdl = o.use_pdl != 0;
    c->prefill_gemm = o.prefill_gemm != 0;
    c->tp_rank = o.tp_rank;
    c->tp_size = o.tp_size < 1 ? 1 : o.tp_size;
    c->nccl = o.nccl_comm;
    c->dim = g.dim; c->hidden = g.hidden; c->n_layers = g.n_layers; c->n_heads = g.n_heads; c->n_kv = g.n_kv;
    c->hd = g.dim / g.n_heads; c->vocab = g.vocab; c->theta = g.theta; c->eps = g.eps; c->bos = g.bos; c->eos = g.eos;
    // --context default 65536, capped at 131072 (mistral/mistral_infer.m:518-523)
    c->max_seq = o.max_seq > 0 ? o.max_seq : 65536;
    if (c->max_seq > 131072) c->max_seq = 131072;
    c->MB = (o.max_batch > 0 && o.max_batch <= kMaxS) ? o.max_batch : kMaxS;
    auto bail = [&](int code) { sd_ctx_free(c); return code; };
    if (c->hd != 128) return bail(fail(SD_ERR_UNSUPPORTED, "head_dim %d (kernels are built for 128)", c->hd));
    if (c->n_heads % c->n_kv || c->n_heads / c->n_kv != 4)
        return bail(fail(SD_ERR_UNSUPPORTED, "GQA ratio %d:%d (kernels are built for 4:1)", c->n_heads, c->n_kv));
    if (c->n_kv % c->tp_size || c->hidden % (c->tp_size * 32) || c->tp_rank < 0 || c->tp_rank >= c->tp_size)
        return bail(fail(SD_ERR_INVALID, "tp %d/%d does not divide the model", c->tp_rank, c->tp_size));
    if (c->tp_size > 1 && !c->nccl) return bail(fail(SD_ERR_INVALID, "tp_size > 1 needs an NCCL communicator"));
    c->nkv_l = c->n_kv / c->tp_size;
    c->nh_l = c->nkv_l * 4;
    c->q_rows = c->nh_l * c->hd;
    c->kv_rows = c->nkv_l * c->hd;
    c->qkv_rows = c->q_rows + 2 * c->kv_rows;
    c->hid_l = c->hidden / c->tp_size;
    if (c->dim % 1024 || c->dim > 4096 || c->q_rows % 128 || c->hid_l % 128)
        return bail(fail(SD_ERR_UNSUPPORTED, "dim %d must be a multiple of 1024 (<= 4096), local q rows %d and hidden %d of 128",
                         c->dim, c->q_rows, c->hid_l));
    if (cudaSetDevice(c->dev) != cudaSuccess) return bail(fail(SD_ERR_INVALID, "bad device %d", c->dev));
    if ((rc = ck(cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking), "stream"))) return bail(rc);
    if ((rc = gemv_prepare_device(c->dev))) return bail(rc);

    // ---- weights ----
    size_t stage_bytes = 0;
    for (auto& t : g.t)
        if (t.type == 2) stage_bytes = std::max(stage_bytes, (size_t)(t.ne[0] * t.ne[1] / 32 * 18));
    uint8_t* staging = nullptr;
    if ((rc = dalloc(&staging, stage_bytes))) return bail(rc);
    auto cleanup_stage = [&]() { cudaFree(staging); };
    c->L.resize(c->n_layers);
    const int r0q = c->tp_rank * c->q_rows, r0kv = c->tp_rank * c->kv_rows, r0h = c->tp_rank * c->hid_l;
    for (int l = 0; l < c->n_layers && !rc; ++l) {
        LayerW& W = c->L[l];
        char nm[128];
        auto T = [&](const char* f) {
            snprintf(nm, sizeof nm, f, l);
            return g.find(nm);
        };
        size_t b;
        b = qmat_bytes(c->qkv_rows, c->dim);
        if ((rc = dalloc(&W.qkv, b, &c->weight_bytes))) break;
        cudaMemset(W.qkv, 0, b);
        if ((rc = upload_q4(c, g, T("blk.%d.attn_q.weight"), r0q, c->q_rows, 0, c->dim, RowMap{c->q_rows, 0, 0}, W.qkv, staging, stage_bytes))) break;
        if ((rc = upload_q4(c, g, T("blk.%d.attn_k.weight"), r0kv, c->kv_rows, 0, c->dim, RowMap{c->kv_rows, 0, c->q_rows}, W.qkv, staging, stage_bytes))) break;
        if ((rc = upload_q4(c, g, T("blk.%d.attn_v.weight"), r0kv, c->kv_rows, 0, c->dim, RowMap{c->kv_rows, 0, c->q_rows + c->kv_rows}, W.qkv, staging, stage_bytes))) break;
        b = qmat_bytes(c->dim, c->q_rows);
        if ((rc = dalloc(&W.wo, b, &c->weight_bytes))) break;
        cudaMemset(W.wo, 0, b);
        if ((rc = upload_q4(c, g, T("blk.%d.attn_output.weight"), 0, c->dim, r0q / 32, c->q_rows, RowMap{c->dim, 0, 0}, W.wo, staging, stage_bytes))) break;
        b = qmat_bytes(2 * c->hid_l, c->dim);
        if ((rc = dalloc(&W.w13, b, &c->weight_bytes))) break;
        cudaMemset(W.w13, 0, b);
        // gate rows -> row-groups 4u, 4u+1 ; up rows -> 4u+2, 4u+3 (units of 32 hidden units)
        if ((rc = upload_q4(c, g, T("blk.%d.ffn_gate.weight"), r0h, c->hid_l, 0, c->dim, RowMap{32, 64, 0}, W.w13, staging, stage_bytes))) break;
        if ((rc = upload_q4(c, g, T("blk.%d.ffn_up.weight"), r0h, c->hid_l, 0, c->dim, RowMap{32, 64, 32}, W.w13, staging, stage_bytes))) break;
        b = qmat_bytes(c->dim, c->hid_l);
        if ((rc = dalloc(&W.w2, b, &c->weight_bytes))) break;
        cudaMemset(W.w2, 0, b);
        if ((rc = upload_q4(c, g, T("blk.%d.ffn_down.weight"), 0, c->dim, r0h / 32, c->hid_l, RowMap{c->dim, 0, 0}, W.w2, staging, stage_bytes))) break;
        snprintf(nm, sizeof nm, "blk.%d.attn_norm.weight", l);
        if ((rc = upload_f32(c, g, nm, &W.rms_att, c->dim))) break;
        snprintf(nm, sizeof nm, "blk.%d.ffn_norm.weight", l);
        if ((rc = upload_f32(c, g, nm, &W.rms_ffn, c->dim))) break;
    }
    if (!rc) {
        const GTensor* te = g.find("token_embd.weight");
        const GTensor* tl = g.find("output.weight");
        // the embedding may be Q4_0 or Q4_K, the LM head Q4_0, Q6_K (the real Mistral Q4_0 files) or Q4_K
        // (mistral/mistral_model.h:125-157, :1110-1122); every layer matrix is Q4_0
        if (!te || (te->type != 2 && te->type != 12) || !tl || (tl->type != 2 && tl->type != 12 && tl->type != 14))
            rc = fail(SD_ERR_FORMAT, "token_embd must be Q4_0 or Q4_K and output Q4_0, Q4_K or Q6_K");
        else if ((te->type == 12 || tl->type != 2) && c->dim % 256)
            rc = fail(SD_ERR_FORMAT, "K-quant tensors need dim %% 256 == 0");
        if (!rc) {
            c->embd_type = (int)te->type;
            size_t eb = te->type == 2 ? (size_t)c->vocab * c->dim / 32 * 18 : (size_t)c->vocab * c->dim / 256 * 144;
            if (!(rc = dalloc(&c->embd, eb, &c->weight_bytes)))
                rc = ck(cudaMemcpy(c->embd, g.base + te->off, eb, cudaMemcpyHostToDevice), "embedding upload");
        }
        if (!rc && tl->type == 2) {
            size_t b = qmat_bytes(c->vocab, c->dim);
            if (!(rc = dalloc(&c->lm, b, &c->weight_bytes))) {
                cudaMemset(c->lm, 0, b);
                rc = upload_q4(c, g, tl, 0, c->vocab, 0, c->dim, RowMap{c->vocab, 0, 0}, c->lm, staging, stage_bytes);
            }
        } else if (!rc) {
            c->lm_type = (int)tl->type;
            const size_t n_blocks = (size_t)c->vocab * (c->dim / 256);
            const size_t b = (size_t)c->vocab * kq_device_row_bytes(c->lm_type, c->dim);
            if (!(rc = dalloc(&c->lm, b, &c->weight_bytes)) && !(rc = dalloc(&c->xn, (size_t)c->MB * c->dim))) {
                if (c->lm_type == 12) {
                    rc = ck(cudaMemcpy(c->lm, g.base + tl->off, b, cudaMemcpyHostToDevice), "LM head upload");
                } else {
                    uint8_t* raw = nullptr;
                    if (!(rc = dalloc(&raw, n_blocks * kQ6KBytes))) {
                        rc = ck(cudaMemcpy(raw, g.base + tl->off, n_blocks * kQ6KBytes, cudaMemcpyHostToDevice),
                                "LM head upload");
                        if (!rc) rc = ck(launch_repack_q6k(raw, c->lm, n_blocks, c->st), "Q6_K repack");
                        if (!rc) rc = ck(cudaStreamSynchronize(c->st), "Q6_K repack");
                        cudaFree(raw);
                    }
                }
            }
        }
        if (!rc) rc = upload_f32(c, g, "output_norm.weight", &c->rms_final, c->dim);
    }
    cleanup_stage();
    if (rc) return bail(rc);
    // RoPE inverse frequencies on the host (mistral/mistral_model.h:69-74)
    {
        std::vector<float> th(c->hd / 2);
        for (int i = 0; i < c->hd / 2; ++i) th[i] = 1.0f / powf(c->theta, (2.0f * (float)i) / (float)c->hd);
        if ((rc = dalloc(&c->theta_inv, th.size()))) return bail(rc);
        if ((rc = ck(cudaMemcpy(c->theta_inv, th.data(), th.size() * 4, cudaMemcpyHostToDevice), "theta"))) return bail(rc);
    }
    // ---- KV ring + buffers ----
    const size_t kvn = (size_t)c->n_layers * c->max_seq * c->kv_rows;
    if ((rc = dalloc(&c->kc, kvn, &c->kv_bytes)) || (rc = dalloc(&c->vc, kvn, &c->kv_bytes))) return bail(rc);
    cudaMemset(c->kc, 0, kvn * 2);
    cudaMemset(c->vc, 0, kvn * 2);
    const int MB = c->MB;
    const int amax = std::max(c->dim, c->q_rows);
    // split-K chunk of the attention: short rings favour parallelism, long ones fewer partials
    c->attn_chunk = c->max_seq <= 8192 ? 32 : (c->max_seq <= 32768 ? 64 : 128);
    c->max_chunks = (c->max_seq + c->attn_chunk - 1) / c->attn_chunk;
    if ((rc = dalloc(&c->x, (size_t)MB * c->dim)) || (rc = dalloc(&c->y, (size_t)c->ypart_max * MB * c->dim)) ||
        (rc = dalloc(&c->act.qs, (size_t)MB * amax)) || (rc = dalloc(&c->act.d, (size_t)MB * amax / 32)) ||
        (rc = dalloc(&c->act.sum, (size_t)MB * amax / 32)) || (rc = dalloc(&c->hact.qs, (size_t)MB * c->hid_l)) ||
        (rc = dalloc(&c->hact.d, (size_t)MB * c->hid_l / 32)) || (rc = dalloc(&c->hact.sum, (size_t)MB * c->hid_l / 32)) ||
        (rc = dalloc(&c->q, (size_t)MB * c->q_rows)) ||
        (rc = dalloc(&c->part_ml, (size_t)MB * c->nh_l * c->max_chunks)) ||
        (rc = dalloc(&c->part_acc, (size_t)MB * c->nh_l * c->max_chunks * 128)) ||
        (rc = dalloc(&c->logits, (size_t)kMaxVerify * c->vocab)) || (rc = dalloc(&c->probs, (size_t)c->vocab)) ||
        (rc = dalloc(&c->argmax, kMaxVerify)) || (rc = dalloc(&c->ctrl_sub, kMaxVerify)) || (rc = dalloc(&c->ctrl, 1)) || (rc = dalloc(&c->dctrl, 1)) ||
        (rc = dalloc(&c->err, 1)) || (rc = dalloc(&c->gs, 1)))
        return bail(rc);
    cudaMemset(c->err, 0, sizeof(int));
    cudaMemset(c->x, 0, (size_t)MB * c->dim * 4);
    cudaMemset(c->y, 0, (size_t)c->ypart_max * MB * c->dim * 4);
    if ((rc = ck(cudaMallocHost(&c->gs_h, sizeof(GenState)), "pinned")))
        return bail(rc);
    if (c->tp_size > 1) {
        c->tp_buf = (size_t)c->ypart_max * MB * c->dim;
        const size_t bytes = 2 * c->tp_buf * sizeof(float) + kMaxTp * sizeof(unsigned long long);
        if ((rc = ck(cudaMalloc(&c->tp_mem, bytes), "cudaMalloc")) || (rc = ck(cudaMemset(c->tp_mem, 0, bytes), "memset")) ||
            (rc = dalloc(&c->tp_base, 1)) || (rc = ck(cudaMemset(c->tp_base, 0, sizeof(unsigned long long)), "memset")))
            return bail(rc);
    }
    if (o.forward_kernel && (rc = setup_fused(c))) return bail(rc);
    if ((rc = ck(cudaDeviceSynchronize(), "context build"))) return bail(rc);
    *out = c;
    return SD_OK;
}

int sd_gguf_describe(const void* gguf_base, size_t gguf_len, sd_gguf_desc* out) {
    clear_error();
    if (!gguf_base || !out) return fail(SD_ERR_INVALID, "sd_gguf_describe: null argument");
    GGUF g;
    int rc = gguf_parse(gguf_base, gguf_len, g);
    if (rc) return rc;
    memset(out, 0, sizeof(*out));
    out->version = g.version;
    out->n_tensors = (uint32_t)g.t.size();
    out->dim = g.dim;
    out->hidden_dim = g.hidden;
    out->n_layers = g.n_layers;
    out->n_heads = g.n_heads;
    out->n_kv_heads = g.n_kv;
    out->head_dim = g.dim / g.n_heads;
    out->vocab_size = g.vocab;
    out->context_length = g.ctx_len;
    out->rope_theta = g.theta;
    out->rms_eps = g.eps;
    out->bos_id = g.bos;
    out->eos_id = g.eos;
    out->data_offset = g.data_start;
    return SD_OK;
}

int sd_ctx_create(const void* gguf_base, size_t gguf_len, const sd_ctx_opts* opts, sd_ctx** out) {
    return ctx_build(gguf_base, gguf_len, opts, out);
}

int sd_ctx_create_file(const char* path, const sd_ctx_opts* opts, sd_ctx** out) {
    clear_error();
    if (!path || !out) return fail(SD_ERR_INVALID, "null argument");
    int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(SD_ERR_INVALID, "cannot open %s", path);
    struct stat stt;
    if (fstat(fd, &stt) != 0) {
        close(fd);
        return fail(SD_ERR_INVALID, "cannot stat %s", path);
    }
    void* base = mmap(nullptr, stt.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (base == MAP_FAILED) return fail(SD_ERR_OOM, "mmap %s failed", path);
    int rc = ctx_build(base, stt.st_size, opts, out);
    munmap(base, stt.st_size);
    return rc;
}

int sd_ctx_info(const sd_ctx* c, sd_model_info* o) {
    if (!c || !o) return fail(SD_ERR_INVALID, "null argument");
    o->dim = c->dim; o->hidden_dim = c->hidden; o->n_layers = c->n_layers; o->n_heads = c->n_heads;
    o->n_kv_heads = c->n_kv; o->head_dim = c->hd; o->vocab_size = c->vocab; o->max_seq = c->max_seq;
    o->rope_theta = c->theta; o->rms_eps = c->eps; o->bos_id = c->bos; o->eos_id = c->eos;
    o->tp_rank = c->tp_rank; o->tp_size = c->tp_size; o->weight_bytes = c->weight_bytes; o->kv_bytes = c->kv_bytes;
    o->forward_kernel = (c->fused && (c->tp_size == 1 || c->tpx.n > 1)) ? 1 : 0;
    return SD_OK;
}

int sd_ctx_device_error(sd_ctx* c) {
    if (!c) return fail(SD_ERR_INVALID, "null context");
    cudaSetDevice(c->dev);
    int h = 0;
    if (cudaMemcpyAsync(&h, c->err, sizeof(int), cudaMemcpyDeviceToHost, c->st) != cudaSuccess ||
        cudaStreamSynchronize(c->st) != cudaSuccess)
        return fail(SD_ERR_CUDA, "reading device error word");
    cudaMemsetAsync(c->err, 0, sizeof(int), c->st);
    cudaStreamSynchronize(c->st);
    return h;
}

void* sd_ctx_stream(sd_ctx* c) { return c ? (void*)c->st : nullptr; }

int sd_ctx_tp_handle(sd_ctx* c, void* out) {
    clear_error();
    if (!c || !out) return fail(SD_ERR_INVALID, "null argument");
    if (c->tp_size <= 1 || !c->tp_mem) return fail(SD_ERR_INVALID, "not a tensor-parallel context");
    cudaSetDevice(c->dev);
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, c->tp_mem), "cudaIpcGetMemHandle");
    memcpy(out, &h, sizeof(h));
    return SD_OK;
}

int sd_ctx_tp_connect(sd_ctx* c, const void* handles, int n) {
    clear_error();
    if (!c || !handles) return fail(SD_ERR_INVALID, "null argument");
    if (c->tp_size <= 1 || n != c->tp_size || n > kMaxTp) return fail(SD_ERR_INVALID, "need %d handles", c->tp_size);
    if (c->tpx.n > 1) return fail(SD_ERR_INVALID, "peers already connected");
    cudaSetDevice(c->dev);
    CK(cudaStreamSynchronize(c->st), "sync");
    TpXchg t{};
    t.n = n;
    t.rank = c->tp_rank;
    t.base = c->tp_base;
    t.buf = c->tp_buf;
    for (int r = 0; r < n; ++r) {
        void* p = c->tp_mem;
        if (r != c->tp_rank) {
            cudaIpcMemHandle_t h;
            memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)r * sizeof(h), sizeof(h));
            cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) {
                for (void* q : c->tp_opened) cudaIpcCloseMemHandle(q);
                c->tp_opened.clear();
                return cuda_fail(e, "cudaIpcOpenMemHandle");
            }
            c->tp_opened.push_back(p);
        }
        t.y[r] = static_cast<float*>(p);
        t.flags[r] = reinterpret_cast<unsigned long long*>(static_cast<float*>(p) + 2 * c->tp_buf);
    }
    c->tpx = t;
    // forwards captured for the NCCL path are rebuilt on next use
    for (auto* gs : {c->fwd_graph, c->fwd_graph_kv})
        for (int i = 0; i <= kMaxVerify; ++i)
            if (gs[i]) {
                cudaGraphExecDestroy(gs[i]);
                gs[i] = nullptr;
            }
    if (c->iter_graph) {
        cudaGraphExecDestroy(c->iter_graph);
        c->iter_graph = nullptr;
        for (int& k : c->iter_key) k = -1;
    }
    return SD_OK;
}

int sd_forward_dev(sd_ctx* c, const int32_t* tokens_dev, int S, int pos, float* logits_dev, int32_t* argmax_dev, void* stream) {
    clear_error();
    if (!c || !tokens_dev || S < 1 || S > kMaxVerify || pos < 0) return fail(SD_ERR_INVALID, "sd_forward_dev: bad arguments");
    if (pos + S > c->max_seq) return fail(SD_ERR_INVALID, "positions past the KV ring (%d)", c->max_seq);
    cudaSetDevice(c->dev);
    cudaEvent_t ev;
    if (stream) {
        // order after the caller's stream
        CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "event");
        CK(cudaEventRecord(ev, (cudaStream_t)stream), "event");
        CK(cudaStreamWaitEvent(c->st, ev, 0), "event");
        cudaEventDestroy(ev);
    }
    int rc = set_ctrl(c, c->ctrl, tokens_dev, S, pos, false);
    if (rc) return rc;
    if ((rc = run_forward(c, S))) return rc;
    if (logits_dev) CK(cudaMemcpyAsync(logits_dev, c->logits, (size_t)S * c->vocab * 4, cudaMemcpyDeviceToDevice, c->st), "logits");
    if (argmax_dev) CK(cudaMemcpyAsync(argmax_dev, c->argmax, (size_t)S * 4, cudaMemcpyDeviceToDevice, c->st), "argmax");
    if (stream) {
        CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "event");
        CK(cudaEventRecord(ev, c->st), "event");
        CK(cudaStreamWaitEvent((cudaStream_t)stream, ev, 0), "event");
        cudaEventDestroy(ev);
    }
    return SD_OK;
}

int sd_forward(sd_ctx* c, const int32_t* tokens, int S, int pos, float* logits, int32_t* argmax) {
    clear_error();
    if (!c || !tokens || S < 1 || S > kMaxVerify || pos < 0) return fail(SD_ERR_INVALID, "sd_forward: bad arguments");
    if (pos + S > c->max_seq) return fail(SD_ERR_INVALID, "positions past the KV ring (%d)", c->max_seq);
    int rc = check_tokens(c, tokens, S);
    if (rc) return rc;
    cudaSetDevice(c->dev);
    if ((rc = set_ctrl(c, c->ctrl, tokens, S, pos, true))) return rc;
    if ((rc = run_forward(c, S))) return rc;
    if (logits) CK(cudaMemcpyAsync(logits, c->logits, (size_t)S * c->vocab * 4, cudaMemcpyDeviceToHost, c->st), "logits");
    if (argmax) CK(cudaMemcpyAsync(argmax, c->argmax, (size_t)S * 4, cudaMemcpyDeviceToHost, c->st), "argmax");
    return finish(c);
}

int sd_forward_layers(sd_ctx* c, int n_layers, const int32_t* tokens, int S, int pos, float* logits, int32_t* argmax) {
    clear_error();
    if (!c || !tokens || S < 1 || S > kMaxVerify || pos < 0 || n_layers < 1 || n_layers > c->n_layers)
        return fail(SD_ERR_INVALID, "sd_forward_layers: bad arguments");
    if (pos + S > c->max_seq) return fail(SD_ERR_INVALID, "positions past the KV ring");
    int rc = check_tokens(c, tokens, S);
    if (rc) return rc;
    cudaSetDevice(c->dev);
    if ((rc = set_ctrl(c, c->ctrl, tokens, S, pos, true))) return rc;
    if ((rc = enqueue_forward(c, S, n_layers, c->kc, c->vc, c->ctrl, true))) return rc;
    if (logits) CK(cudaMemcpyAsync(logits, c->logits, (size_t)S * c->vocab * 4, cudaMemcpyDeviceToHost, c->st), "logits");
    if (argmax) CK(cudaMemcpyAsync(argmax, c->argmax, (size_t)S * 4, cudaMemcpyDeviceToHost, c->st), "argmax");
    return finish(c);
}

// Single-op model layer (kernel-per-op path, single-GPU contexts).  x travels through c->x; ctrl carries the
// position, the token (embedding) and the valid count.
static int single_op_ready(sd_ctx* c, const char* what) {
    if (!c) return fail(SD_ERR_INVALID, "%s: null context", what);
    if (c->tp_size > 1) return fail(SD_ERR_UNSUPPORTED, "%s: single-GPU contexts only", what);
    cudaSetDevice(c->dev);
    return SD_OK;
}

int sd_embed_token(sd_ctx* c, int token, float* out) {
    clear_error();
    int rc = single_op_ready(c, "sd_embed_token");
    if (rc) return rc;
    if (!out) return fail(SD_ERR_INVALID, "sd_embed_token: null output");
    if ((rc = check_tokens(c, &token, 1))) return rc;
    if ((rc = set_ctrl(c, c->ctrl, &token, 1, 0, true))) return rc;
    NormArgs na = norm_args(c, 1, c->ctrl);
    CK(launch_norm_quant(0, na, c->st, false), "embed");
    CK(cudaMemcpyAsync(out, c->x, (size_t)c->dim * 4, cudaMemcpyDeviceToHost, c->st), "download");
    return finish(c);
}

int sd_layer_decode(sd_ctx* c, float* x, int layer, int pos) {
    clear_error();
    int rc = single_op_ready(c, "sd_layer_decode");
    if (rc) return rc;
    if (!x || layer < 0 || layer >= c->n_layers || pos < 0 || pos >= c->max_seq)
        return fail(SD_ERR_INVALID, "sd_layer_decode: bad arguments");
    const int32_t tok = 0;
    if ((rc = set_ctrl(c, c->ctrl, &tok, 1, pos, true))) return rc;
    CK(cudaMemcpyAsync(c->x, x, (size_t)c->dim * 4, cudaMemcpyHostToDevice, c->st), "upload");
    NormArgs na = norm_args(c, 1, c->ctrl);
    na.w = c->L[layer].rms_att;
    CK(launch_norm_quant(2, na, c->st, false), "norm");
    const float* w_next = layer + 1 < c->n_layers ? c->L[layer + 1].rms_att : c->rms_final;
    if ((rc = enqueue_layer_perop(c, layer, 1, c->kc, c->vc, c->ctrl, na, w_next))) return rc;
    CK(cudaMemcpyAsync(x, c->x, (size_t)c->dim * 4, cudaMemcpyDeviceToHost, c->st), "download");
    return finish(c);
}

int sd_logits(sd_ctx* c, const float* x, int S, float* logits) {
    clear_error();
    int rc = single_op_ready(c, "sd_logits");
    if (rc) return rc;
    if (!x || !logits || S < 1 || S > c->MB) return fail(SD_ERR_INVALID, "sd_logits: bad arguments (S <= %d)", c->MB);
    int32_t toks[kMaxS] = {0};
    if ((rc = set_ctrl(c, c->ctrl, toks, S, 0, true))) return rc;
    CK(cudaMemcpyAsync(c->x, x, (size_t)S * c->dim * 4, cudaMemcpyHostToDevice, c->st), "upload");
    NormArgs na = norm_args(c, S, c->ctrl);
    na.w = c->rms_final;
    CK(launch_norm_quant(2, na, c->st, false), "final norm");
    if ((rc = enqueue_head_perop(c, S, c->ctrl, 0))) return rc;
    CK(cudaMemcpyAsync(logits, c->logits, (size_t)S * c->vocab * 4, cudaMemcpyDeviceToHost, c->st), "download");
    return finish(c);
}

// Prompt tokens [0, n) at start_pos .. into the ring through the batched engine's GEMMs: 64 slices of 8 tokens per
// forward (M = 512 on the tcgen05 GEMM), so every weight tile read from HBM serves 512 tokens instead of 8.
// *used = false (and nothing enqueued) when the prompt is short, the option is off or the batched engine does not
// serve this model (tensor parallelism, K-quant embedding or LM head).
namespace {

constexpr int kGemmPrefillMin = 256;
constexpr int kPrefillSlices = 64;

int gemm_prefill(sd_ctx* c, const int32_t* tokens, int n, int start_pos, bool* used) {
    *used = false;
    if (!c->prefill_gemm || c->pf_unsupported || n < kGemmPrefillMin || c->tp_size > 1 || c->lm_type != 2 ||
        c->embd_type != 2)
        return SD_OK;
    if (!c->pf) {
        const int rc = batch_create_prefill(c, kPrefillSlices, kMaxS, c->kc, c->vc, c->max_seq, c->st, &c->pf);
        if (rc == SD_ERR_UNSUPPORTED) {
            c->pf_unsupported = true;
            clear_error();
            return SD_OK;
        }
        if (rc) return rc;
    }
    const int rc = batch_prefill_ring(c->pf, tokens, n, start_pos);
    if (!rc) *used = true;
    return rc;
}

}  // namespace

int sd_prefill(sd_ctx* c, const int32_t* tokens, int n, int start_pos) {
    clear_error();
    if (!c || !tokens || n < 0 || start_pos < 0) return fail(SD_ERR_INVALID, "sd_prefill: bad arguments");
    if (start_pos + n > c->max_seq) return fail(SD_ERR_INVALID, "prompt past the KV ring");
    int rc = check_tokens(c, tokens, n);
    if (rc) return rc;
    cudaSetDevice(c->dev);
    bool gemm = false;
    if ((rc = gemm_prefill(c, tokens, n, start_pos, &gemm))) return rc;
    for (int i = gemm ? n : 0; i < n; i += c->MB) {
        const int S = std::min(c->MB, n - i);
        if ((rc = set_ctrl(c, c->ctrl, tokens + i, S, start_pos + i, true))) return rc;
        if ((rc = run_forward(c, S, false))) return rc;
    }
    return finish(c);
}

int sd_kv_read(sd_ctx* c, int layer, int pos0, int n, uint16_t* k, uint16_t* v) {
    clear_error();
    if (!c || layer < 0 || layer >= c->n_layers || pos0 < 0 || n < 0 || pos0 + n > c->max_seq)
        return fail(SD_ERR_INVALID, "sd_kv_read: bad arguments");
    cudaSetDevice(c->dev);
    const size_t off = ((size_t)layer * c->max_seq + pos0) * c->kv_rows;
    if (k) CK(cudaMemcpyAsync(k, c->kc + off, (size_t)n * c->kv_rows * 2, cudaMemcpyDeviceToHost, c->st), "kv read");
    if (v) CK(cudaMemcpyAsync(v, c->vc + off, (size_t)n * c->kv_rows * 2, cudaMemcpyDeviceToHost, c->st), "kv read");
    return finish(c);
}

int sd_ngram_draft(const int32_t* history, int hlen, int ngram_n, int max_draft, int current, int32_t* draft_out, int* match_pos) {
    clear_error();
    if ((hlen > 0 && !history) || hlen < 0 || ngram_n < 1 || max_draft < 0 || (max_draft > 0 && !draft_out))
        return fail(SD_ERR_INVALID, "sd_ngram_draft: bad arguments");
    if (sd_device_count() == 0) return fail(SD_ERR_NO_DEVICE, "no CUDA device");
    int* dh = nullptr;
    int* dout = nullptr;
    cudaStream_t st = nullptr;
    int rc = SD_OK;
    if ((rc = ck(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "stream"))) return rc;
    if (!(rc = dalloc(&dh, (size_t)std::max(hlen, 1))) && !(rc = dalloc(&dout, (size_t)max_draft + 2))) {
        if (hlen > 0) rc = ck(cudaMemcpyAsync(dh, history, (size_t)hlen * 4, cudaMemcpyHostToDevice, st), "upload");
        if (!rc) rc = ck(launch_ngram_scan(dh, hlen, ngram_n, max_draft, current, dout, st), "ngram");
        std::vector<int> h(max_draft + 2);
        if (!rc) rc = ck(cudaMemcpyAsync(h.data(), dout, (max_draft + 2) * 4, cudaMemcpyDeviceToHost, st), "download");
        if (!rc) rc = ck(cudaStreamSynchronize(st), "ngram");
        if (!rc) {
            for (int i = 0; i < h[0]; ++i) draft_out[i] = h[2 + i];
            if (match_pos) *match_pos = h[1];
            rc = h[0];
        }
    }
    cudaFree(dh);
    cudaFree(dout);
    cudaStreamDestroy(st);
    return rc;
}

int sd_spec_accept(sd_ctx* c, const float* draft_probs, const float* logits, const int32_t* draft, int n_draft, float temp,
                   int bonus_mode, uint64_t seed, uint64_t* counter, int32_t* accepted) {
    clear_error();
    if (!c || !logits || !draft || !accepted || n_draft < 1 || n_draft > kMaxVerify - 1 || (temp > 0 && !draft_probs))
        return fail(SD_ERR_INVALID, "sd_spec_accept: bad arguments");
    cudaSetDevice(c->dev);
    int rc = check_tokens(c, draft, n_draft);
    if (rc) return rc;
    // scratch: logits rows in c->logits, probs in c->probs, small arrays in the tail of c->y
    int* d_draft = reinterpret_cast<int*>(c->y);
    float* d_dp = reinterpret_cast<float*>(c->y) + 16;
    int* d_acc = reinterpret_cast<int*>(c->y) + 32;
    int* d_n = reinterpret_cast<int*>(c->y) + 48;
    unsigned long long* d_ctr = reinterpret_cast<unsigned long long*>(c->y + 64);
    unsigned long long ctr = counter ? *counter : 0;
    CK(cudaMemcpyAsync(c->logits, logits, (size_t)(n_draft + 1) * c->vocab * 4, cudaMemcpyHostToDevice, c->st), "upload");
    CK(cudaMemcpyAsync(d_draft, draft, n_draft * 4, cudaMemcpyHostToDevice, c->st), "upload");
    if (draft_probs) CK(cudaMemcpyAsync(d_dp, draft_probs, n_draft * 4, cudaMemcpyHostToDevice, c->st), "upload");
    else CK(cudaMemsetAsync(d_dp, 0, n_draft * 4, c->st), "memset");
    CK(cudaMemcpyAsync(d_ctr, &ctr, 8, cudaMemcpyHostToDevice, c->st), "upload");
    CK(launch_spec_accept(c->logits, c->probs, d_draft, d_dp, n_draft, c->vocab, temp, bonus_mode, seed, d_ctr, d_acc, d_n,
                          c->st), "spec_accept");
    int na = 0;
    CK(cudaMemcpyAsync(&na, d_n, 4, cudaMemcpyDeviceToHost, c->st), "download");
    CK(cudaMemcpyAsync(&ctr, d_ctr, 8, cudaMemcpyDeviceToHost, c->st), "download");
    CK(cudaStreamSynchronize(c->st), "spec_accept");
    if (na < 1 || na > n_draft + 1) return fail(SD_ERR_CUDA, "spec_accept returned %d", na);
    CK(cudaMemcpy(accepted, d_acc, na * 4, cudaMemcpyDeviceToHost), "download");
    if (counter) *counter = ctr;
    return na;
}

int sd_sample_token(sd_ctx* c, float* logits, int n, float temp, int top_k, float top_p, float rep_penalty,
                    const int32_t* prev_tokens, int n_prev, uint64_t seed, uint64_t* counter) {
    clear_error();
    constexpr int kMaxPrev = 4096;
    if (!c || !logits || n < 1 || n > c->vocab || n_prev < 0 || n_prev > kMaxPrev || (n_prev > 0 && !prev_tokens))
        return fail(SD_ERR_INVALID, "sd_sample_token: bad arguments (n <= vocab, n_prev <= %d)", kMaxPrev);
    if (temp > 0 && top_k > kMaxTopK)
        return fail(SD_ERR_INVALID, "sd_sample_token: top_k %d above the device limit %d", top_k, kMaxTopK);
    cudaSetDevice(c->dev);
    // scratch: the row in c->logits, its copy in c->probs, prev tokens / result / counter in c->y
    int* d_prev = reinterpret_cast<int*>(c->y);
    int* d_out = reinterpret_cast<int*>(c->y) + kMaxPrev;
    unsigned long long* d_ctr = reinterpret_cast<unsigned long long*>(c->y + kMaxPrev + 4);
    unsigned long long ctr = counter ? *counter : 0;
    GenParamsDev p{};
    p.temp = temp;
    p.top_k = top_k;
    p.top_p = top_p;
    p.rep_penalty = rep_penalty;
    CK(cudaMemcpyAsync(c->logits, logits, (size_t)n * 4, cudaMemcpyHostToDevice, c->st), "upload");
    if (n_prev > 0) CK(cudaMemcpyAsync(d_prev, prev_tokens, (size_t)n_prev * 4, cudaMemcpyHostToDevice, c->st), "upload");
    CK(cudaMemcpyAsync(d_ctr, &ctr, 8, cudaMemcpyHostToDevice, c->st), "upload");
    CK(launch_sample_token(c->logits, c->probs, n, p, d_prev, n_prev, seed, d_ctr, d_out, c->st), "sample_token");
    int tok = -1;
    CK(cudaMemcpyAsync(&tok, d_out, 4, cudaMemcpyDeviceToHost, c->st), "download");
    CK(cudaMemcpyAsync(&ctr, d_ctr, 8, cudaMemcpyDeviceToHost, c->st), "download");
    CK(cudaMemcpyAsync(logits, c->logits, (size_t)n * 4, cudaMemcpyDeviceToHost, c->st), "download");
    CK(cudaStreamSynchronize(c->st), "sample_token");
    if (tok < 0 || tok >= n) return fail(SD_ERR_CUDA, "sample_token returned %d", tok);
    if (counter) *counter = ctr;
    return tok;
}

int sd_spec_softmax(sd_ctx* c, const float* logits, float* probs, int n, float temp) {
    clear_error();
    if (!c || !logits || !probs || n < 1 || n > c->vocab) return fail(SD_ERR_INVALID, "sd_spec_softmax: bad arguments");
    cudaSetDevice(c->dev);
    CK(cudaMemcpyAsync(c->logits, logits, (size_t)n * 4, cudaMemcpyHostToDevice, c->st), "upload");
    CK(launch_spec_softmax(c->logits, c->probs, n, temp, c->st), "spec_softmax");
    CK(cudaMemcpyAsync(probs, c->probs, (size_t)n * 4, cudaMemcpyDeviceToHost, c->st), "download");
    CK(cudaStreamSynchronize(c->st), "spec_softmax");
    return SD_OK;
}

int sd_spec_sample_probs(sd_ctx* c, const float* probs, int n, uint64_t seed, uint64_t* counter) {
    clear_error();
    if (!c || !probs || n < 1 || n > c->vocab) return fail(SD_ERR_INVALID, "sd_spec_sample_probs: bad arguments");
    cudaSetDevice(c->dev);
    int* d_out = reinterpret_cast<int*>(c->y);
    unsigned long long* d_ctr = reinterpret_cast<unsigned long long*>(c->y + 4);
    unsigned long long ctr = counter ? *counter : 0;
    CK(cudaMemcpyAsync(c->probs, probs, (size_t)n * 4, cudaMemcpyHostToDevice, c->st), "upload");
    CK(cudaMemcpyAsync(d_ctr, &ctr, 8, cudaMemcpyHostToDevice, c->st), "upload");
    CK(launch_spec_sample_probs(c->probs, n, seed, d_ctr, d_out, c->st), "spec_sample_probs");
    int tok = -1;
    CK(cudaMemcpyAsync(&tok, d_out, 4, cudaMemcpyDeviceToHost, c->st), "download");
    CK(cudaMemcpyAsync(&ctr, d_ctr, 8, cudaMemcpyDeviceToHost, c->st), "download");
    CK(cudaStreamSynchronize(c->st), "spec_sample_probs");
    if (tok < 0 || tok >= n) return fail(SD_ERR_CUDA, "spec_sample_probs returned %d", tok);
    if (counter) *counter = ctr;
    return tok;
}

void sd_gen_params_default(sd_gen_params* p) {
    if (!p) return;
    memset(p, 0, sizeof(*p));
    // mistral/mistral_infer.m:396-410 defaults
    p->mode = SD_GEN_GREEDY;
    p->max_tokens = 128;
    p->temp = 0.7f;
    p->top_p = 0.9f;
    p->top_k = 40;
    p->rep_penalty = 1.1f;
    p->rep_window = 64;
    p->spec_k = 4;
    p->ngram_n = 3;
    p->draft_layers = 8;
    p->history_has_current = 0;
    p->bonus_mode = SD_BONUS_ARGMAX;
    p->seed = 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Generation loops
// ---------------------------------------------------------------------------------------------
namespace {

int ensure_gen_buffers(sd_ctx* c, int cap) {
    if (c->g_cap >= cap) return SD_OK;
    cudaFree(c->g_out);
    cudaFree(c->g_hist);
    c->g_out = c->g_hist = nullptr;
    c->g_cap = 0;
    int rc = dalloc(&c->g_out, (size_t)cap);
    if (!rc) rc = dalloc(&c->g_hist, (size_t)cap);
    if (!rc) c->g_cap = cap;
    return rc;
}

int ensure_draft_kv(sd_ctx* c, int layers) {
    if (c->draft_layers_alloc >= layers) return SD_OK;
    cudaFree(c->dkc);
    cudaFree(c->dvc);
    c->dkc = c->dvc = nullptr;
    c->draft_layers_alloc = 0;
    c->draft_kv_hist = c->draft_kv_layers = 0;
    const size_t n = (size_t)layers * c->max_seq * c->kv_rows;
    int rc = dalloc(&c->dkc, n);
    if (!rc) rc = dalloc(&c->dvc, n);
    if (rc) return rc;
    cudaMemset(c->dkc, 0, n * 2);
    cudaMemset(c->dvc, 0, n * 2);
    c->draft_layers_alloc = layers;
    return SD_OK;
}

// One decode iteration, enqueued on c->st (captured into c->iter_graph).
int enqueue_iteration(sd_ctx* c, const GenParamsDev& p, int K, int draft_layers) {
    int rc;
    if (p.mode == SD_MODE_SELF) {
        CK(launch_gen_self_begin(c->gs, c->dctrl, c->st), "self begin");
        for (int k = 0; k < K; ++k) {
            if ((rc = enqueue_forward(c, 1, draft_layers, c->dkc, c->dvc, c->dctrl, true))) return rc;
            CK(launch_gen_draft_step(c->gs, c->dctrl, c->argmax, k, c->st), "draft step");
        }
        CK(launch_gen_self_verify(c->gs, c->ctrl, K, c->st), "self verify");
        if ((rc = enqueue_forward(c, K + 1, c->n_layers, c->kc, c->vc, c->ctrl, true))) return rc;
    } else {
        const int S = p.mode == SD_MODE_NGRAM ? K + 1 : 1;
        CK(launch_gen_prepare(c->gs, c->ctrl, p, c->st), "prepare");
        if ((rc = enqueue_forward(c, S, c->n_layers, c->kc, c->vc, c->ctrl, true))) return rc;
    }
    CK(launch_gen_commit(c->gs, c->ctrl, c->logits, c->probs, c->argmax, p, c->vocab, c->st), "commit");
    return SD_OK;
}

int iteration_graph(sd_ctx* c, const GenParamsDev& p, int K, int draft_layers) {
    // key: mode, K, draft depth, and whether sampling parameters change kernel arguments (captured by value)
    const int key[6] = {p.mode, K, draft_layers, (int)(p.temp * 1e4f), p.top_k, (int)(p.rep_penalty * 1e4f)};
    bool same = c->iter_graph != nullptr;
    for (int i = 0; i < 6; ++i) same = same && key[i] == c->iter_key[i];
    // any other captured parameter change forces a rebuild
    same = same && memcmp(&c->iter_p, &p, sizeof p) == 0;
    if (same) return SD_OK;
    if (c->iter_graph) {
        cudaGraphExecDestroy(c->iter_graph);
        c->iter_graph = nullptr;
    }
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(c->st, cudaStreamCaptureModeThreadLocal), "capture");
    int rc = enqueue_iteration(c, p, K, draft_layers);
    cudaError_t e = cudaStreamEndCapture(c->st, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return cuda_fail(e, "end capture");
    e = cudaGraphInstantiate(&c->iter_graph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(e, "graph instantiate");
    memcpy(c->iter_key, key, sizeof key);
    c->iter_p = p;
    return SD_OK;
}

double now_ms() {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

}  // namespace

extern "C" {

int sd_decode(sd_ctx* c, const sd_gen_params* gp, const int32_t* history, int n_hist, int first_token, int32_t* out_tokens,
              int out_cap, sd_gen_stats* stats) {
    clear_error();
    if (!c || !gp || !history || n_hist < 1 || !out_tokens || out_cap < 1) return fail(SD_ERR_INVALID, "sd_decode: bad arguments");
    if (first_token < 0 || first_token >= c->vocab) return fail(SD_ERR_INVALID, "bad first token");
    int rc = check_tokens(c, history, n_hist);
    if (rc) return rc;
    const int mode = gp->mode == SD_GEN_NGRAM ? SD_MODE_NGRAM : gp->mode == SD_GEN_SELF_SPEC ? SD_MODE_SELF : SD_MODE_GREEDY;
    int K = gp->spec_k < 1 ? 1 : gp->spec_k;
    if (mode != SD_MODE_GREEDY && K + 1 > kMaxVerify)
        return fail(SD_ERR_UNSUPPORTED, "spec_k %d needs %d tokens per verify (at most %d)", K, K + 1, kMaxVerify);
    int dl = gp->draft_layers < 1 ? 1 : gp->draft_layers;
    if (dl >= c->n_layers) dl = c->n_layers - 1;
    if (mode == SD_MODE_SELF && dl < 1) return fail(SD_ERR_INVALID, "self-speculation needs >= 2 layers");
    cudaSetDevice(c->dev);
    const int cap = n_hist + gp->max_tokens + 2 * kMaxVerify + 16;
    if ((rc = ensure_gen_buffers(c, cap))) return rc;
    if (mode == SD_MODE_SELF && (rc = ensure_draft_kv(c, dl))) return rc;
    // the first token counts as generated (printed before the loop, mistral_infer.m:615-621)
    GenParamsDev p{};
    p.mode = mode;
    p.temp = gp->temp;
    p.top_k = gp->top_k;
    p.top_p = gp->top_p;
    p.rep_penalty = gp->rep_penalty;
    p.rep_window = gp->rep_window;
    p.ignore_eos = gp->ignore_eos;
    p.eos_id = c->eos;
    p.spec_k = K;
    p.ngram_n = gp->ngram_n < 1 ? 3 : gp->ngram_n;
    p.history_has_current = gp->history_has_current;
    p.bonus_mode = gp->bonus_mode == SD_BONUS_REFERENCE ? SD_BONUS_REF_UNIFORM : SD_BONUS_ARGMAX_FIXED;
    // greedy loop runs max_tokens more tokens (mistral_infer.m:690-716); the speculative loops run
    // until max_tokens - 1 (speculative.h:232, mistral_infer.m:652-654)
    p.gen_limit = mode == SD_MODE_GREEDY ? gp->max_tokens : gp->max_tokens - 1;
    p.max_seq = c->max_seq;
    GenState h{};
    h.cur = first_token;
    h.pos = n_hist - 1;  // history = prompt + first token; the first token sits at position n_prompt
    h.done = p.gen_limit <= 0 || (!p.ignore_eos && first_token == c->eos);
    h.out_cap = cap;
    h.out = c->g_out;
    h.hist_cap = cap;
    h.hist = c->g_hist;
    h.hlen = n_hist;
    h.seed = gp->seed;
    h.rng_counter = c->rng_start;  // continues the Philox stream after the first-token sample
    c->rng_start = 1ull << 20;
    *c->gs_h = h;
    CK(cudaMemcpyAsync(c->g_hist, history, (size_t)n_hist * 4, cudaMemcpyHostToDevice, c->st), "history");
    CK(cudaMemcpyAsync(c->gs, c->gs_h, sizeof(GenState), cudaMemcpyHostToDevice, c->st), "state");
    if (mode == SD_MODE_SELF && !(gp->reuse_draft_kv && c->draft_kv_hist >= n_hist - 1 && c->draft_kv_layers == dl)) {
        // drafter KV prefill through the first dl layers (mistral_infer.m:675-681)
        c->draft_kv_hist = 0;
        for (int i = 0; i < n_hist - 1; i += c->MB) {
            const int S = std::min(c->MB, n_hist - 1 - i);
            if ((rc = set_ctrl(c, c->dctrl, history + i, S, i, true))) return rc;
            if ((rc = enqueue_forward(c, S, dl, c->dkc, c->dvc, c->dctrl, false))) return rc;
        }
        c->draft_kv_hist = n_hist - 1;
        c->draft_kv_layers = dl;
    }
    if ((rc = iteration_graph(c, p, K, dl))) return rc;
    const double t0 = now_ms();
    int generated = 0;
    int guard = 0;
    while (!c->gs_h->done) {
        // launch at least as many iterations as tokens remaining / tokens per iteration (lower bound)
        const int per = mode == SD_MODE_GREEDY ? 1 : K + 1;
        int batch = std::max(1, (p.gen_limit - generated) / per);
        if (batch > 64) batch = 64;
        for (int i = 0; i < batch; ++i) CK(cudaGraphLaunch(c->iter_graph, c->st), "iteration");
        CK(cudaMemcpyAsync(c->gs_h, c->gs, sizeof(GenState), cudaMemcpyDeviceToHost, c->st), "state");
        CK(cudaStreamSynchronize(c->st), "decode");
        generated = c->gs_h->generated;
        if (++guard > 1000000) return fail(SD_ERR_TIMEOUT, "decode did not terminate");
    }
    const double t1 = now_ms();
    if ((rc = check_device_error(c->err, c->st))) return rc;
    GenState& s = *c->gs_h;
    const int n = std::min(s.n_out, out_cap);
    if (n > 0) CK(cudaMemcpy(out_tokens, c->g_out, (size_t)n * 4, cudaMemcpyDeviceToHost), "download");
    if (stats) {
        stats->n_generated = s.n_out;
        stats->total_draft = s.total_draft;
        stats->total_accepted = s.total_accepted;
        stats->total_iterations = s.total_iterations;
        stats->ms_decode = t1 - t0;
    }
    return n;
}

int sd_generate(sd_ctx* c, const sd_gen_params* gp, const int32_t* prompt, int n_prompt, int32_t* out_tokens, int out_cap,
                sd_gen_stats* stats) {
    clear_error();
    if (!c || !gp || !prompt || n_prompt < 1 || !out_tokens || out_cap < 1) return fail(SD_ERR_INVALID, "sd_generate: bad arguments");
    // room for the last verify batch (as the decode loop's stop rule)
    const int vw = std::max(kMaxS, (gp->mode == SD_GEN_GREEDY ? 0 : std::max(gp->spec_k, 1)) + 1);
    if (n_prompt + gp->max_tokens + vw + 1 > c->max_seq) return fail(SD_ERR_INVALID, "prompt + tokens exceed the KV ring");
    int rc = check_tokens(c, prompt, n_prompt);
    if (rc) return rc;
    cudaSetDevice(c->dev);
    const double t0 = now_ms();
    // prefill: all but the last chunk through the GEMMs when the prompt is long, the rest in W4A8 chunks of
    // max_batch tokens; logits of the last prompt token
    const int tail = (n_prompt - 1) % c->MB + 1;
    bool gemm = false;
    if ((rc = gemm_prefill(c, prompt, n_prompt - tail, 0, &gemm))) return rc;
    for (int i = gemm ? n_prompt - tail : 0; i < n_prompt; i += c->MB) {
        const int S = std::min(c->MB, n_prompt - i);
        if ((rc = set_ctrl(c, c->ctrl, prompt + i, S, i, true))) return rc;
        if ((rc = run_forward(c, S, i + S >= n_prompt))) return rc;  // logits of the last chunk only
    }
    const int last = (n_prompt - 1) % c->MB;
    // first token: sample_token with repetition penalty over the prompt window (mistral_infer.m:610-621)
    std::vector<int32_t> hist(prompt, prompt + n_prompt);
    int first;
    {
        GenParamsDev p{};
        p.mode = SD_MODE_GREEDY;
        p.temp = gp->temp;
        p.top_k = gp->top_k;
        p.top_p = gp->top_p;
        p.rep_penalty = gp->rep_penalty;
        p.rep_window = gp->rep_window;
        p.ignore_eos = 1;
        p.eos_id = c->eos;
        p.gen_limit = 1;
        p.max_seq = c->max_seq;
        const int cap = n_prompt + gp->max_tokens + 2 * kMaxVerify + 16;
        if ((rc = ensure_gen_buffers(c, cap))) return rc;
        GenState h{};
        h.cur = 0;
        h.pos = n_prompt;
        h.out_cap = cap;
        h.out = c->g_out;
        h.hist_cap = cap;
        h.hist = c->g_hist;
        h.hlen = n_prompt;
        h.seed = gp->seed;
        h.rng_counter = 0;
        h.n_draft = 0;
        *c->gs_h = h;
        CK(cudaMemcpyAsync(c->g_hist, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, c->st), "history");
        CK(cudaMemcpyAsync(c->gs, c->gs_h, sizeof(GenState), cudaMemcpyHostToDevice, c->st), "state");
        // commit samples from logits row 0: move the last prompt row there
        if (last != 0)
            CK(cudaMemcpyAsync(c->logits, c->logits + (size_t)last * c->vocab, (size_t)c->vocab * 4, cudaMemcpyDeviceToDevice, c->st), "logits");
        CK(launch_gen_commit(c->gs, c->ctrl, c->logits, c->probs, c->argmax, p, c->vocab, c->st), "first token");
        CK(cudaMemcpyAsync(c->gs_h, c->gs, sizeof(GenState), cudaMemcpyDeviceToHost, c->st), "state");
        CK(cudaStreamSynchronize(c->st), "first token");
        CK(cudaMemcpy(&first, c->g_out, 4, cudaMemcpyDeviceToHost), "first token");
        c->rng_start = c->gs_h->rng_counter;
    }
    const double t1 = now_ms();
    hist.push_back(first);
    std::vector<int32_t> rest(std::max(out_cap, 1));
    sd_gen_stats st2{};
    int n = sd_decode(c, gp, hist.data(), (int)hist.size(), first, rest.data(), (int)rest.size(), &st2);
    if (n < 0) return n;
    out_tokens[0] = first;
    const int m = std::min(n, out_cap - 1);
    for (int i = 0; i < m; ++i) out_tokens[1 + i] = rest[i];
    if (stats) {
        *stats = st2;
        stats->n_generated = 1 + st2.n_generated;
        stats->ms_prefill = t1 - t0;
    }
    return 1 + m;
}

}  // extern "C"

int sd_ctx_model_view(sd_ctx* c, ModelView* m) {
    if (!c || !m) return fail(SD_ERR_INVALID, "model view: bad arguments");
    if (c->n_layers > kMaxLayers) return fail(SD_ERR_UNSUPPORTED, "more than %d layers", kMaxLayers);
    *m = ModelView{};
    m->dev = c->dev;
    m->tp_size = c->tp_size;
    m->dim = c->dim;
    m->hidden = c->hid_l;
    m->n_layers = c->n_layers;
    m->n_heads = c->nh_l;
    m->n_kv = c->nkv_l;
    m->hd = c->hd;
    m->vocab = c->vocab;
    m->eos = c->eos;
    m->eps = c->eps;
    m->q_rows = c->q_rows;
    m->kv_rows = c->kv_rows;
    m->qkv_rows = c->qkv_rows;
    for (int l = 0; l < c->n_layers; ++l) {
        m->qkv[l] = c->L[l].qkv;
        m->wo[l] = c->L[l].wo;
        m->w13[l] = c->L[l].w13;
        m->w2[l] = c->L[l].w2;
        m->rms_att[l] = c->L[l].rms_att;
        m->rms_ffn[l] = c->L[l].rms_ffn;
    }
    m->embd = c->embd;
    m->embd_type = c->embd_type;
    m->lm = c->lm;
    m->lm_type = c->lm_type;
    m->rms_final = c->rms_final;
    m->theta_inv = c->theta_inv;
    m->err = c->err;
    return SD_OK;
}
