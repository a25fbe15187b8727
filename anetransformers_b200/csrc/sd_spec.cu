// sd_spec.cu -- on-device sampling, n-gram drafting and speculative acceptance.
//
//   k_argmax        sample_argmax        mistral/mistral_model.h:1136-1143 (first index on ties)
//   k_sample_token  sample_token         mistral/mistral_model.h:1145-1240 (rep penalty, temperature,
//                                        top-k, top-p, linear-CDF draw)
//   k_ngram_draft   ngram_draft_fn       mistral/speculative.h:425-464 (earliest exact match)
//   k_spec_accept   spec_accept          mistral/speculative.h:121-198 (greedy / Leviathan rule) plus
//                   the callers' bonus override (speculative.h:312-317, mistral_infer.m:332-337)
//   k_gen_*         the per-iteration bookkeeping of the decode loops (mistral_infer.m:252-391,
//                   690-716; speculative.h:217-379): history, output, position, stats, stop
//
// Random numbers: the reference draws (float)arc4random()/(float)UINT32_MAX; here the 32-bit draws
// come from Philox4x32-10 (Salmon et al. 2011) keyed by the seed, draw k = word 0 of counter k, the
// same stream the CPU oracle uses, so given equal logits the same uniforms are consumed in order.
#include "sd_common.cuh"
#include "sd_spec.h"

namespace sd {

__device__ __forceinline__ uint32_t philox_u32(uint64_t seed, uint64_t counter) {
    uint32_t c0 = (uint32_t)counter, c1 = (uint32_t)(counter >> 32), c2 = 0, c3 = 0;
    uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
        const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0;
        c1 = lo1;
        c2 = n2;
        c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c0;
}

__device__ __forceinline__ float rng_uniform(GenState* g) {
    const uint32_t u = philox_u32(g->seed, g->rng_counter++);
    return (float)u / (float)0xFFFFFFFFu;
}

// ---------------------------------------------------------------------------------------------
// Block reductions (1024 threads)
// ---------------------------------------------------------------------------------------------
constexpr int kSampleThreads = 1024;

// (value, index) max with the smallest index winning ties.
__device__ __forceinline__ void argmax_merge(float& v, int& i, float v2, int i2) {
    if (v2 > v || (v2 == v && i2 < i)) {
        v = v2;
        i = i2;
    }
}

__device__ void block_argmax(float& v, int& i) {
    __shared__ float sv[32];
    __shared__ int si[32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) argmax_merge(v, i, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, i, o));
    __syncthreads();
    if (lane == 0) {
        sv[w] = v;
        si[w] = i;
    }
    __syncthreads();
    if (w == 0) {
        v = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
        i = lane < (int)(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            argmax_merge(v, i, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, i, o));
        if (lane == 0) {
            sv[0] = v;
            si[0] = i;
        }
    }
    __syncthreads();
    v = sv[0];
    i = si[0];
}

__device__ float block_sum(float v) {
    __shared__ float s[32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) s[w] = v;
    __syncthreads();
    float r = 0.f;
    if (w == 0) {
        r = lane < (int)(blockDim.x >> 5) ? s[lane] : 0.f;
        r = warp_sum(r);
        if (lane == 0) s[0] = r;
    }
    __syncthreads();
    r = s[0];
    return r;
}

__device__ float block_max(float v) {
    __shared__ float s[32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) s[w] = v;
    __syncthreads();
    float r = -INFINITY;
    if (w == 0) {
        r = lane < (int)(blockDim.x >> 5) ? s[lane] : -INFINITY;
        r = warp_max(r);
        if (lane == 0) s[0] = r;
    }
    __syncthreads();
    r = s[0];
    return r;
}

__device__ int block_argmax_row(const float* x, int n) {
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int j = threadIdx.x; j < n; j += blockDim.x) argmax_merge(v, idx, x[j], j);
    block_argmax(v, idx);
    return idx;
}

// First index i with r < cumsum(p[0..i]) over n probabilities (linear-CDF draw of
// speculative.h:60-68 / mistral_model.h:1227-1234); n-1 if r is never reached.  Each thread owns a
// contiguous range; range sums are scanned, then the owning thread walks its range in order.
__device__ int block_cdf_draw(const float* p, int n, float r, float scale) {
    __shared__ float part[kSampleThreads];
    __shared__ int found;
    const int per = (n + blockDim.x - 1) / blockDim.x;
    const int j0 = threadIdx.x * per, j1 = min(n, j0 + per);
    float s = 0.f;
    for (int j = j0; j < j1; ++j) s += p[j] * scale;
    part[threadIdx.x] = s;
    if (threadIdx.x == 0) found = n - 1;
    __syncthreads();
    if (threadIdx.x == 0) {  // exclusive scan in order (1024 adds)
        float c = 0.f;
        for (int k = 0; k < (int)blockDim.x; ++k) {
            const float v = part[k];
            part[k] = c;
            c += v;
        }
    }
    __syncthreads();
    float c = part[threadIdx.x];
    bool done = false;
    for (int j = j0; j < j1 && !done; ++j) {
        c += p[j] * scale;
        if (r < c) {
            atomicMin(&found, j);
            done = true;
        }
    }
    __syncthreads();
    return found;
}

// ---------------------------------------------------------------------------------------------
__global__ void k_argmax(const float* __restrict__ logits, int vocab, int S, int* __restrict__ out, const DevCtrl* ctrl) {
    if (ctrl && ctrl->done) return;
    pdl_trigger();
    pdl_wait();
    const int nv = ctrl ? min(ctrl->n_valid, S) : S;
    const int s = blockIdx.x;
    if (s >= nv) return;
    const int idx = block_argmax_row(logits + (size_t)s * vocab, vocab);
    if (threadIdx.x == 0) out[s] = idx;
}

cudaError_t launch_argmax(const float* logits, int vocab, int S, int* out, const DevCtrl* ctrl, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S);
    cfg.blockDim = dim3(kSampleThreads);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_argmax, logits, vocab, S, out, ctrl);
}

// Argmax from the (logit, row) keys the persistent forward's LM head reduces: row = ~low word.
__global__ void k_argmax_keys(const unsigned long long* __restrict__ keys, int S, int* __restrict__ out, const DevCtrl* ctrl) {
    if (ctrl && ctrl->done) return;
    const int nv = ctrl ? min(ctrl->n_valid, S) : S;
    const int s = threadIdx.x;
    if (s < nv) out[s] = (int)(0xFFFFFFFFu - (uint32_t)(keys[s] & 0xFFFFFFFFull));
}

cudaError_t launch_argmax_keys(const unsigned long long* keys, int S, int* out, const DevCtrl* ctrl, cudaStream_t st) {
    k_argmax_keys<<<1, 32, 0, st>>>(keys, S, out, ctrl);
    return cudaGetLastError();
}

// sample_token on logits row `row` (modified in place: repetition penalty, top-k selection marks).
// Thread 0 performs the sequential parts exactly as the reference orders them.
__device__ int sample_token_dev(float* logits, int n, const GenParamsDev& p, const int* prev, int n_prev, GenState* g) {
    __shared__ int s_tok;
    __shared__ float tk_v[kMaxTopK];
    __shared__ int tk_i[kMaxTopK];
    // repetition penalty, once per occurrence in the window (mistral_model.h:1147-1158)
    if (threadIdx.x == 0 && p.rep_penalty != 1.0f && n_prev > 0) {
        for (int i = 0; i < n_prev; ++i) {
            const int t = prev[i];
            if (t < 0 || t >= n) continue;
            if (logits[t] > 0) logits[t] /= p.rep_penalty;
            else logits[t] *= p.rep_penalty;
        }
    }
    __syncthreads();
    if (p.temp <= 0.f) return block_argmax_row(logits, n);
    int top_k = p.top_k > 0 ? p.top_k : 40;
    if (top_k > n) top_k = n;
    if (top_k > kMaxTopK) top_k = kMaxTopK;
    // top-k values in descending order (ties: smallest index first)
    for (int k = 0; k < top_k; ++k) {
        float v = -INFINITY;
        int idx = 0x7fffffff;
        for (int j = threadIdx.x; j < n; j += blockDim.x) argmax_merge(v, idx, logits[j], j);
        block_argmax(v, idx);
        if (threadIdx.x == 0) {
            tk_v[k] = v;
            tk_i[k] = idx;
            logits[idx] = -INFINITY;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        // tempered softmax over top-k, nucleus cut, renormalise, linear CDF (mistral_model.h:1201-1234)
        float pr[kMaxTopK];
        const float mx = tk_v[0];
        float sum = 0.f;
        for (int i = 0; i < top_k; ++i) {
            pr[i] = expf((tk_v[i] - mx) / p.temp);
            sum += pr[i];
        }
        for (int i = 0; i < top_k; ++i) pr[i] /= sum;
        int eff = top_k;
        if (p.top_p > 0.f && p.top_p < 1.0f) {
            float cum = 0.f;
            for (int i = 0; i < top_k; ++i) {
                cum += pr[i];
                if (cum >= p.top_p) {
                    eff = i + 1;
                    break;
                }
            }
            sum = 0.f;
            for (int i = 0; i < eff; ++i) sum += pr[i];
            for (int i = 0; i < eff; ++i) pr[i] /= sum;
        }
        const float r = rng_uniform(g);
        float cdf = 0.f;
        int res = tk_i[0];
        for (int i = 0; i < eff; ++i) {
            cdf += pr[i];
            if (r < cdf) {
                res = tk_i[i];
                break;
            }
        }
        s_tok = res;
    }
    __syncthreads();
    return s_tok;
}

// spec_softmax of one logits row into probs (speculative.h:37-57); returns nothing, probs written.
__device__ void spec_softmax_dev(const float* l, float* probs, int n, float temperature) {
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < n; j += blockDim.x) mx = fmaxf(mx, l[j]);
    mx = block_max(mx);
    const float inv_t = temperature > 0.f ? 1.0f / temperature : 0.0f;
    float s = 0.f;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const float e = expf((l[j] - mx) * inv_t);
        probs[j] = e;
        s += e;
    }
    s = block_sum(s);
    const float inv = 1.0f / s;
    for (int j = threadIdx.x; j < n; j += blockDim.x) probs[j] = probs[j] * inv;
    __syncthreads();
}

// ---------------------------------------------------------------------------------------------
// Generation bookkeeping.  GenState lives in device memory; one CTA of 1024 threads.
// ---------------------------------------------------------------------------------------------
__device__ void emit(GenState* g, int tok) {
    if (g->n_out < g->out_cap) g->out[g->n_out] = tok;
    g->n_out++;
    if (g->hlen < g->hist_cap) g->hist[g->hlen] = tok;
    g->hlen++;
}

// Draft phase.  NGRAM: prompt-lookup scan (speculative.h:425-464) over the history (excluding the
// current token unless the reference wiring is requested); writes the verify batch
// [current, drafts...] into ctrl.  GREEDY / no draft: batch = [current].
__device__ void gen_prepare_body(GenState* g, DevCtrl* ctrl, const GenParamsDev& p) {
    __shared__ int best;
    if (g->done) {
        if (threadIdx.x == 0) {
            ctrl->n_valid = 0;
            ctrl->done = 1;
        }
        return;
    }
    const int cur = g->cur;
    int nd = 0;
    if (p.mode == SD_MODE_NGRAM) {
        const int n = p.ngram_n;
        const int hlen = min(p.history_has_current ? g->hlen : g->hlen - 1, g->hist_cap);
        const int* h = g->hist;
        if (threadIdx.x == 0) best = 0x7fffffff;
        __syncthreads();
        if (hlen >= n) {
            const int plen = n > 16 ? 16 : n;
            // pattern = history[hlen-plen+1 .. hlen-1] ++ [cur]
            for (int i = threadIdx.x; i <= hlen - plen - 1; i += blockDim.x) {
                bool ok = true;
                for (int j = 0; j < plen && ok; ++j) {
                    const int pj = (j == plen - 1) ? cur : h[hlen - plen + 1 + j];
                    ok = (h[i + j] == pj);
                }
                if (ok) atomicMin(&best, i);
            }
            __syncthreads();
            if (best != 0x7fffffff) {
                const int m = best + plen;
                nd = min(p.spec_k, hlen - m);
                if (threadIdx.x < nd) ctrl->tokens[1 + threadIdx.x] = h[m + threadIdx.x];
            }
        }
    }
    if (threadIdx.x == 0) {
        ctrl->tokens[0] = cur;
        ctrl->n_valid = 1 + nd;
        ctrl->pos = g->pos;
        ctrl->done = 0;
        g->n_draft = nd;
        for (int i = 0; i < nd; ++i) g->draft_probs[i] = 0.9f;   // n-gram "probability"
    }
}

__global__ void k_gen_prepare(GenState* g, DevCtrl* ctrl, GenParamsDev p) { gen_prepare_body(g, ctrl, p); }

// Batched streams: CTA b prepares stream b.
__global__ void k_bgen_prepare(GenState* gs, DevCtrl* ctrls, GenParamsDev p) {
    gen_prepare_body(gs + blockIdx.x, ctrls + blockIdx.x, p);
}

// Self-speculative drafter step: after a draft-depth forward of token tokens[0] at pos + k, take the
// argmax as draft k (speculative.h:524-535; draft_probs = 1) and feed it as the next draft input.
__global__ void k_gen_draft_step(GenState* g, DevCtrl* dctrl, const int* argmax, int k) {
    if (g->done) return;
    if (threadIdx.x == 0) {
        const int nx = argmax[0];
        g->drafts[k] = nx;
        g->draft_probs[k] = 1.0f;
        dctrl->tokens[0] = nx;
        dctrl->pos = g->pos + k + 1;
        dctrl->n_valid = 1;
    }
}

// Self-spec: set up the draft chain (token cur at pos) and, after the K draft steps, the verify batch.
__global__ void k_gen_self_begin(GenState* g, DevCtrl* dctrl) {
    if (threadIdx.x != 0) return;
    if (g->done) {
        dctrl->n_valid = 0;
        dctrl->done = 1;
        return;
    }
    dctrl->tokens[0] = g->cur;
    dctrl->pos = g->pos;
    dctrl->n_valid = 1;
    dctrl->done = 0;
}

__global__ void k_gen_self_verify(GenState* g, DevCtrl* ctrl, int K) {
    if (threadIdx.x != 0) return;
    if (g->done) {
        ctrl->n_valid = 0;
        ctrl->done = 1;
        return;
    }
    ctrl->tokens[0] = g->cur;
    for (int i = 0; i < K; ++i) ctrl->tokens[1 + i] = g->drafts[i];
    ctrl->n_valid = 1 + K;
    ctrl->pos = g->pos;
    ctrl->done = 0;
    g->n_draft = K;
}

// Accept / emit phase after the verify (or single) forward.  logits: [n_valid][vocab].
__device__ void gen_commit_body(GenState* g, DevCtrl* ctrl, float* logits, float* probs, const int* argmax,
                                const GenParamsDev& p, int vocab) {
    __shared__ int acc[kMaxVerify + 1];
    __shared__ int n_acc_s;
    if (g->done) return;
    const int nd = g->n_draft;
    const int tid = threadIdx.x;
    if (nd == 0) {
        // no draft: single forward + sample_token with repetition penalty over the history window
        // (mistral_infer.m:284-313; greedy loop :691-715)
        const int hs = g->hlen > p.rep_window ? g->hlen - p.rep_window : 0;
        const int n_prev = min(g->hlen, g->hist_cap) - hs;
        const int tok = sample_token_dev(logits, vocab, p, g->hist + hs, n_prev > 0 ? n_prev : 0, g);
        if (tid == 0) {
            acc[0] = tok;
            n_acc_s = 1;
        }
        __syncthreads();
    } else if (p.temp <= 0.f) {
        // greedy acceptance (speculative.h:127-150) on the argmax of each verify row
        if (tid == 0) {
            int na = nd + 1;
            for (int i = 0; i < nd; ++i) {
                const int t = argmax[i];
                acc[i] = t;
                if (t != ctrl->tokens[1 + i]) {
                    na = i + 1;
                    break;
                }
            }
            if (na == nd + 1) {
                // bonus: argmax of the last row (fixed), or the reference's draw from
                // spec_softmax(logits[nd], temp=0) = uniform
                if (p.bonus_mode == SD_BONUS_REF_UNIFORM) {
                    // spec_softmax with inv_t = 0 gives probs = 1 * (1/sum) with sum = vocab; the
                    // reference then walks the CDF sequentially (speculative.h:44-68)
                    const float r = rng_uniform(g);
                    const float inv = 1.0f / (float)vocab;
                    float cdf = 0.f;
                    int b = vocab - 1;
                    for (int j = 0; j < vocab; ++j) {
                        cdf += inv;
                        if (r < cdf) {
                            b = j;
                            break;
                        }
                    }
                    acc[nd] = b;
                } else {
                    acc[nd] = argmax[nd];
                }
            }
            n_acc_s = na;
        }
        __syncthreads();
    } else {
        // stochastic acceptance (speculative.h:153-197)
        __shared__ float r_s;
        __shared__ int res_s;
        int na = nd + 1;
        for (int i = 0; i < nd; ++i) {
            spec_softmax_dev(logits + (size_t)i * vocab, probs, vocab, p.temp);
            const int tok = ctrl->tokens[1 + i];
            if (tid == 0) {
                const float p_tok = probs[tok], q_tok = g->draft_probs[i];
                const float ap = q_tok > 0.f ? fminf(1.0f, p_tok / q_tok) : 0.0f;
                r_s = rng_uniform(g);
                res_s = (r_s < ap) ? 1 : 0;
            }
            __syncthreads();
            if (res_s) {
                if (tid == 0) acc[i] = tok;
                __syncthreads();
                continue;
            }
            // residual distribution max(0, p - q*1[tok]), normalised (or p if it sums to 0)
            const float q_tok = g->draft_probs[i];
            if (tid == 0) probs[tok] = fmaxf(0.0f, probs[tok] - q_tok);
            __syncthreads();
            float s = 0.f;
            for (int j = tid; j < vocab; j += blockDim.x) s += probs[j];
            s = block_sum(s);
            __shared__ float r2;
            if (tid == 0) r2 = rng_uniform(g);
            __syncthreads();
            int t;
            if (s > 0.f) {
                t = block_cdf_draw(probs, vocab, r2, 1.0f / s);
            } else {
                spec_softmax_dev(logits + (size_t)i * vocab, probs, vocab, p.temp);
                t = block_cdf_draw(probs, vocab, r2, 1.0f);
            }
            if (tid == 0) acc[i] = t;
            na = i + 1;
            __syncthreads();
            break;
        }
        if (na == nd + 1) {
            // bonus from the last verify row (the callers' override, speculative.h:312-317)
            spec_softmax_dev(logits + (size_t)nd * vocab, probs, vocab, p.temp);
            __shared__ float r3;
            if (tid == 0) r3 = rng_uniform(g);
            __syncthreads();
            const int t = block_cdf_draw(probs, vocab, r3, 1.0f);
            if (tid == 0) acc[nd] = t;
        }
        if (tid == 0) n_acc_s = na;
        __syncthreads();
    }
    if (tid == 0) {
        const int na = n_acc_s;
        int stop = 0;
        for (int i = 0; i < na; ++i) {
            emit(g, acc[i]);
            g->generated++;
            if (!p.ignore_eos && acc[i] == p.eos_id) {
                stop = 1;
                break;
            }
        }
        if (nd > 0) {
            g->total_draft += nd;
            g->total_accepted += na;
        }
        g->total_iterations++;
        g->pos += na;
        g->cur = acc[na - 1];
        if (stop || g->generated >= p.gen_limit || g->pos + max(kMaxS, (p.mode == SD_MODE_GREEDY ? 0 : p.spec_k) + 1) >= p.max_seq) g->done = 1;
    }
}

__global__ void __launch_bounds__(kSampleThreads) k_gen_commit(GenState* g, DevCtrl* ctrl, float* logits, float* probs,
                                                               const int* argmax, GenParamsDev p, int vocab) {
    gen_commit_body(g, ctrl, logits, probs, argmax, p, vocab);
}

// Batched streams: CTA b commits stream b from its verify rows b*T + row0 .. of logits / argmax.
__global__ void __launch_bounds__(kSampleThreads) k_bgen_commit(GenState* gs, DevCtrl* ctrls, float* logits, float* probs,
                                                                const int* argmax, GenParamsDev p, int vocab, int T,
                                                                int row0) {
    const int b = blockIdx.x;
    gen_commit_body(gs + b, ctrls + b, logits + ((size_t)b * T + row0) * vocab, probs + (size_t)b * vocab,
                    argmax + (size_t)b * T + row0, p, vocab);
}

// After the first-token commit (one greedy sample from the last prompt row): the decode loop's state, as
// the single-stream path sets it up (the first token sits at position n_prompt, not yet fed).
__global__ void k_bgen_first_fixup(GenState* gs, int n, int gen_limit, int ignore_eos, int eos) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n) return;
    GenState* g = gs + b;
    g->pos -= 1;
    g->generated = 0;
    g->total_draft = g->total_accepted = g->total_iterations = 0;
    g->done = (gen_limit <= 0 || (!ignore_eos && g->cur == eos)) ? 1 : 0;
}

// out[0] = streams done, out[1] = the most tokens a live stream still has to generate.
__global__ void k_bcount_done(const GenState* gs, int n, int gen_limit, int* out) {
    int c = 0, rem = 0;
    for (int b = threadIdx.x; b < n; b += blockDim.x) {
        c += gs[b].done ? 1 : 0;
        if (!gs[b].done) rem = max(rem, gen_limit - gs[b].generated);
    }
    c = (int)block_sum((float)c);  // counts far below 2^24: exact
    rem = (int)block_max((float)rem);
    if (threadIdx.x == 0) {
        out[0] = c;
        out[1] = rem;
    }
}

cudaError_t launch_bgen_prepare(GenState* gs, DevCtrl* ctrls, int n, const GenParamsDev& p, cudaStream_t st) {
    k_bgen_prepare<<<n, 1024, 0, st>>>(gs, ctrls, p);
    return cudaGetLastError();
}

cudaError_t launch_bgen_commit(GenState* gs, DevCtrl* ctrls, int n, float* logits, float* probs, const int* argmax,
                               const GenParamsDev& p, int vocab, int T, int row0, cudaStream_t st) {
    k_bgen_commit<<<n, kSampleThreads, 0, st>>>(gs, ctrls, logits, probs, argmax, p, vocab, T, row0);
    return cudaGetLastError();
}

cudaError_t launch_bgen_first_fixup(GenState* gs, int n, int gen_limit, int ignore_eos, int eos, cudaStream_t st) {
    k_bgen_first_fixup<<<(n + 127) / 128, 128, 0, st>>>(gs, n, gen_limit, ignore_eos, eos);
    return cudaGetLastError();
}

cudaError_t launch_bcount_done(const GenState* gs, int n, int gen_limit, int* out, cudaStream_t st) {
    k_bcount_done<<<1, 256, 0, st>>>(gs, n, gen_limit, out);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// Stand-alone primitives for the C ABI (sd_ngram_draft, sd_spec_accept)
// ---------------------------------------------------------------------------------------------
__global__ void k_ngram_scan(const int* h, int hlen, int n, int max_draft, int cur, int* out /*[1 + max_draft + 1]*/) {
    __shared__ int best;
    if (threadIdx.x == 0) best = 0x7fffffff;
    __syncthreads();
    int nd = 0, m = -1;
    if (hlen >= n) {
        const int plen = n > 16 ? 16 : n;
        for (int i = threadIdx.x; i <= hlen - plen - 1; i += blockDim.x) {
            bool ok = true;
            for (int j = 0; j < plen && ok; ++j) {
                const int pj = (j == plen - 1) ? cur : h[hlen - plen + 1 + j];
                ok = (h[i + j] == pj);
            }
            if (ok) atomicMin(&best, i);
        }
        __syncthreads();
        if (best != 0x7fffffff) {
            m = best + plen;
            nd = min(max_draft, hlen - m);
            for (int i = threadIdx.x; i < nd; i += blockDim.x) out[2 + i] = h[m + i];
        }
    }
    if (threadIdx.x == 0) {
        out[0] = nd;
        out[1] = m;
    }
}

// Stand-alone spec_accept (speculative.h:121-198 + bonus override) for the C ABI: logits [n_draft+1][vocab].
__global__ void __launch_bounds__(kSampleThreads) k_spec_accept(const float* logits, float* probs, const int* draft,
                                                                const float* draft_probs, int nd, int vocab, float temp,
                                                                int bonus_mode, unsigned long long seed,
                                                                unsigned long long* counter, int* accepted, int* n_acc) {
    __shared__ GenState g;
    __shared__ int acc_s[kMaxVerify + 1];
    __shared__ float r_s;
    __shared__ int res_s;
    if (threadIdx.x == 0) {
        g.seed = seed;
        g.rng_counter = *counter;
    }
    __syncthreads();
    const int tid = threadIdx.x;
    int na = nd + 1;
    if (temp <= 0.f) {
        for (int i = 0; i < nd; ++i) {
            const int t = block_argmax_row(logits + (size_t)i * vocab, vocab);
            if (tid == 0) acc_s[i] = t;
            if (t != draft[i]) {
                na = i + 1;
                break;
            }
        }
        if (na == nd + 1) {
            if (bonus_mode == SD_BONUS_REF_UNIFORM) {
                if (tid == 0) {
                    const float r = rng_uniform(&g);
                    const float inv = 1.0f / (float)vocab;
                    float cdf = 0.f;
                    int b = vocab - 1;
                    for (int j = 0; j < vocab; ++j) {
                        cdf += inv;
                        if (r < cdf) {
                            b = j;
                            break;
                        }
                    }
                    acc_s[nd] = b;
                }
            } else {
                const int t = block_argmax_row(logits + (size_t)nd * vocab, vocab);
                if (tid == 0) acc_s[nd] = t;
            }
        }
    } else {
        for (int i = 0; i < nd; ++i) {
            spec_softmax_dev(logits + (size_t)i * vocab, probs, vocab, temp);
            const int tok = draft[i];
            if (tid == 0) {
                const float ap = draft_probs[i] > 0.f ? fminf(1.0f, probs[tok] / draft_probs[i]) : 0.0f;
                r_s = rng_uniform(&g);
                res_s = (r_s < ap) ? 1 : 0;
            }
            __syncthreads();
            if (res_s) {
                if (tid == 0) acc_s[i] = tok;
                __syncthreads();
                continue;
            }
            if (tid == 0) probs[tok] = fmaxf(0.0f, probs[tok] - draft_probs[i]);
            __syncthreads();
            float s = 0.f;
            for (int j = tid; j < vocab; j += blockDim.x) s += probs[j];
            s = block_sum(s);
            if (tid == 0) r_s = rng_uniform(&g);
            __syncthreads();
            int t;
            if (s > 0.f) {
                t = block_cdf_draw(probs, vocab, r_s, 1.0f / s);
            } else {
                spec_softmax_dev(logits + (size_t)i * vocab, probs, vocab, temp);
                t = block_cdf_draw(probs, vocab, r_s, 1.0f);
            }
            if (tid == 0) acc_s[i] = t;
            na = i + 1;
            __syncthreads();
            break;
        }
        if (na == nd + 1) {
            spec_softmax_dev(logits + (size_t)nd * vocab, probs, vocab, temp);
            if (tid == 0) r_s = rng_uniform(&g);
            __syncthreads();
            const int t = block_cdf_draw(probs, vocab, r_s, 1.0f);
            if (tid == 0) acc_s[nd] = t;
        }
    }
    __syncthreads();
    if (tid == 0) {
        for (int i = 0; i < na; ++i) accepted[i] = acc_s[i];
        *n_acc = na;
        *counter = g.rng_counter;
    }
}

cudaError_t launch_spec_accept(const float* logits, float* probs, const int* draft, const float* draft_probs, int n_draft,
                               int vocab, float temp, int bonus_mode, unsigned long long seed,
                               unsigned long long* counter, int* accepted, int* n_acc, cudaStream_t st) {
    k_spec_accept<<<1, kSampleThreads, 0, st>>>(logits, probs, draft, draft_probs, n_draft, vocab, temp, bonus_mode, seed,
                                                counter, accepted, n_acc);
    return cudaGetLastError();
}

// Stand-alone sample_token (mistral/mistral_model.h:1145-1240) for the C ABI.  logits [n] receives the
// repetition penalty in place, as the reference's call does (its later steps leave the array as penalised);
// the top-k selection then runs on the scratch copy.  out[0] = the token; *counter advances by the draws.
__global__ void __launch_bounds__(kSampleThreads) k_sample_token(float* logits, float* scratch, int n, GenParamsDev p,
                                                                 const int* prev, int n_prev, unsigned long long seed,
                                                                 unsigned long long* counter, int* out) {
    __shared__ GenState g;
    if (threadIdx.x == 0) {
        g.seed = seed;
        g.rng_counter = *counter;
        if (p.rep_penalty != 1.0f)
            for (int i = 0; i < n_prev; ++i) {
                const int t = prev[i];
                if (t < 0 || t >= n) continue;
                if (logits[t] > 0) logits[t] /= p.rep_penalty;
                else logits[t] *= p.rep_penalty;
            }
    }
    __syncthreads();
    for (int j = threadIdx.x; j < n; j += blockDim.x) scratch[j] = logits[j];
    __syncthreads();
    GenParamsDev q = p;
    q.rep_penalty = 1.0f;  // applied above
    const int tok = sample_token_dev(scratch, n, q, nullptr, 0, &g);
    if (threadIdx.x == 0) {
        out[0] = tok;
        *counter = g.rng_counter;
    }
}

// spec_softmax (speculative.h:37-57) of one row, and spec_sample_probs (speculative.h:60-68): the linear CDF
// draw of one uniform from (seed, *counter) over probs [n].  out[0] = the drawn index.
__global__ void __launch_bounds__(kSampleThreads) k_spec_softmax(const float* logits, float* probs, int n, float temp) {
    spec_softmax_dev(logits, probs, n, temp);
}

__global__ void __launch_bounds__(kSampleThreads) k_spec_sample_probs(const float* probs, int n, unsigned long long seed,
                                                                      unsigned long long* counter, int* out) {
    __shared__ float r_s;
    if (threadIdx.x == 0) r_s = (float)philox_u32(seed, *counter) / (float)0xFFFFFFFFu;
    __syncthreads();
    const int t = block_cdf_draw(probs, n, r_s, 1.0f);
    if (threadIdx.x == 0) {
        out[0] = t;
        *counter = *counter + 1;
    }
}

cudaError_t launch_sample_token(float* logits, float* scratch, int n, const GenParamsDev& p, const int* prev, int n_prev,
                                unsigned long long seed, unsigned long long* counter, int* out, cudaStream_t st) {
    k_sample_token<<<1, kSampleThreads, 0, st>>>(logits, scratch, n, p, prev, n_prev, seed, counter, out);
    return cudaGetLastError();
}

cudaError_t launch_spec_softmax(const float* logits, float* probs, int n, float temp, cudaStream_t st) {
    k_spec_softmax<<<1, kSampleThreads, 0, st>>>(logits, probs, n, temp);
    return cudaGetLastError();
}

cudaError_t launch_spec_sample_probs(const float* probs, int n, unsigned long long seed, unsigned long long* counter,
                                     int* out, cudaStream_t st) {
    k_spec_sample_probs<<<1, kSampleThreads, 0, st>>>(probs, n, seed, counter, out);
    return cudaGetLastError();
}

cudaError_t launch_ngram_scan(const int* h, int hlen, int n, int max_draft, int cur, int* out, cudaStream_t st) {
    k_ngram_scan<<<1, kSampleThreads, 0, st>>>(h, hlen, n, max_draft, cur, out);
    return cudaGetLastError();
}

cudaError_t launch_gen_prepare(GenState* g, DevCtrl* ctrl, const GenParamsDev& p, cudaStream_t st) {
    k_gen_prepare<<<1, kSampleThreads, 0, st>>>(g, ctrl, p);
    return cudaGetLastError();
}
cudaError_t launch_gen_commit(GenState* g, DevCtrl* ctrl, float* logits, float* probs, const int* argmax,
                              const GenParamsDev& p, int vocab, cudaStream_t st) {
    k_gen_commit<<<1, kSampleThreads, 0, st>>>(g, ctrl, logits, probs, argmax, p, vocab);
    return cudaGetLastError();
}
cudaError_t launch_gen_self_begin(GenState* g, DevCtrl* dctrl, cudaStream_t st) {
    k_gen_self_begin<<<1, 32, 0, st>>>(g, dctrl);
    return cudaGetLastError();
}
cudaError_t launch_gen_draft_step(GenState* g, DevCtrl* dctrl, const int* argmax, int k, cudaStream_t st) {
    k_gen_draft_step<<<1, 32, 0, st>>>(g, dctrl, argmax, k);
    return cudaGetLastError();
}
// Control block of the forward that carries tokens [off, off + kMaxS) of a verify batch.  done is copied
// (it only ever goes 0 -> 1 within a generation, so kernels may read it before their grid dependency
// wait); a slice with no valid token gets n_valid 0.
__global__ void k_ctrl_slice(const DevCtrl* src, DevCtrl* dst, int off) {
    const int i = threadIdx.x;
    if (i < kMaxS) dst->tokens[i] = off + i < kMaxVerify ? src->tokens[off + i] : 0;
    if (i == 0) {
        dst->pos = src->pos + off;
        dst->n_valid = max(src->n_valid - off, 0);
        dst->done = src->done;
    }
}

// Write a control block given by value; tokens_dev (optional) supplies its S tokens from device memory.
__global__ void k_set_ctrl(DevCtrl* dst, DevCtrl val, const int* tokens_dev, int S) {
    const int i = threadIdx.x;
    if (i < kMaxVerify) dst->tokens[i] = (tokens_dev && i < S) ? tokens_dev[i] : val.tokens[i];
    if (i == 0) {
        dst->pos = val.pos;
        dst->n_valid = val.n_valid;
        dst->done = val.done;
    }
}

cudaError_t launch_set_ctrl(DevCtrl* dst, const DevCtrl& val, const int* tokens_dev, int S, cudaStream_t st) {
    k_set_ctrl<<<1, 32, 0, st>>>(dst, val, tokens_dev, S);
    return cudaGetLastError();
}

cudaError_t launch_ctrl_slice(const DevCtrl* src, DevCtrl* dst, int off, cudaStream_t st) {
    k_ctrl_slice<<<1, 32, 0, st>>>(src, dst, off);
    return cudaGetLastError();
}

cudaError_t launch_gen_self_verify(GenState* g, DevCtrl* ctrl, int K, cudaStream_t st) {
    k_gen_self_verify<<<1, 32, 0, st>>>(g, ctrl, K);
    return cudaGetLastError();
}

}  // namespace sd
