// sd_ops.cu -- C ABI of the single-op layer: repacked Q4_0 matrices, Q8_0 quantizer, W4A8 matvec,
// block sums, and the host-pointer drop-ins with the reference's dequant.h signatures.
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "sd_common.cuh"
#include "sd_host.h"
#include "sd_kquant.h"
#include "specdec_b200.h"

using namespace sd;

struct sd_qmat {
    int rows, cols, device;
    uint8_t* w;
    size_t bytes;
};

namespace sd {

static thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(e == cudaErrorMemoryAllocation ? SD_ERR_OOM : SD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

void clear_error() { g_err.clear(); }

int device_sm_count(int dev) {
    static int cache[64] = {0};
    if (dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

int device_max_smem(int dev) {
    static int cache[64] = {0};
    if (dev < 0 || dev >= 64) return 232448;
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || n <= 0)
            n = 232448;
        cache[dev] = n;
    }
    return cache[dev];
}

// Per-device error word for calls that do not belong to a context: a file-scope device variable (zero at
// module load), so neither the word nor reading it allocates.  Its address is looked up once per device with
// that device current; the name itself is only a host-side stand-in in host code.
static __device__ int g_device_err;

int* device_error_word(int dev) {
    static int* words[64] = {nullptr};
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64) return nullptr;
    if (!words[dev]) {
        int prev = -1;
        if (cudaGetDevice(&prev) != cudaSuccess) return nullptr;
        if (prev != dev && cudaSetDevice(dev) != cudaSuccess) return nullptr;
        int* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress((void**)&p, g_device_err);
        if (prev != dev) cudaSetDevice(prev);
        if (e != cudaSuccess) return nullptr;
        words[dev] = p;
    }
    return words[dev];
}

// The single-op device entry points run on the matrix's device; a caller whose current device differs
// would launch on one GPU with another GPU's pointers.
int check_current_device(int dev, const char* what) {
    int cur = -1;
    const cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (cur != dev)
        return fail(SD_ERR_INVALID, "%s: the current device is %d but the matrix lives on device %d", what, cur, dev);
    return SD_OK;
}

int check_device_error(int* word, cudaStream_t st) {
    if (!word) return SD_OK;
    int h = 0;
    cudaError_t e = cudaMemcpyAsync(&h, word, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "reading device error word");
    if (h != 0) {
        cudaMemsetAsync(word, 0, sizeof(int), st);
        return fail(SD_ERR_TIMEOUT, "device wait ran out (device error code %d)", h);
    }
    return SD_OK;
}

// Repack AoS Q4_0 [rows][cols/32] (device) into the tile layout at dst (zero-filled padding rows).
int repack_matrix(const uint8_t* aos_dev, int rows, int cols, RowMap map, uint8_t* dst, cudaStream_t st) {
    cudaError_t e = launch_repack(aos_dev, rows, cols, (size_t)cols / 32 * 18, map, dst, st);
    if (e != cudaSuccess) return cuda_fail(e, "repack");
    return SD_OK;
}

// Once per device (current device): opt every matvec variant into the full shared memory.
int gemv_prepare_device(int dev) {
    static bool done[64] = {false};
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64) return fail(SD_ERR_INVALID, "bad device %d", dev);
    if (done[dev]) return SD_OK;
    cudaError_t e = gemv_init_attrs(device_max_smem(dev));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    done[dev] = true;
    return SD_OK;
}

int gemv_plan(GemvArgs& a, int dev, int* grid_out, size_t* smem_out) {
    if (a.K % 128 != 0 || a.K <= 0) return fail(SD_ERR_INVALID, "matvec: in_dim %d is not a multiple of 128", a.K);
    if (a.S < 1 || a.S > kMaxS) return fail(SD_ERR_INVALID, "matvec: S=%d outside 1..%d", a.S, kMaxS);
    const int max_smem = device_max_smem(dev);
    const int sms = device_sm_count(dev);
    const int want = a.kparts;  // <= 0: choose, 1: forced single slice
    int best = -1;
    for (int kp = 1; kp <= a.nq; ++kp) {
        if (a.nq % kp) continue;
        if (want > 0 && kp != want) continue;
        const int nqp = a.nq / kp, ch = gemv_chunk(nqp);
        if (nqp % ch) continue;
        if (kp > sms) break;
        const int ns = gemv_pick_stages(nqp * 128, a.S, ch, max_smem);
        if (ns >= 3 || (want > 0 && ns >= 2)) {
            best = kp;
            a.chunk = ch;
            a.nstage = ns;
            break;
        }
    }
    if (best < 0) return fail(SD_ERR_INVALID, "matvec: in_dim %d / S=%d has no shared-memory plan", a.K, a.S);
    a.kparts = best;
    *smem_out = gemv_smem_bytes(a.K / best, a.S, a.chunk, a.nstage);
    int grid = sms;
    if (grid > a.n_units * best) grid = a.n_units * best;
    *grid_out = grid;
    return SD_OK;
}

// gemv_plan with the K split fixed for every S (the split chosen at S = kMaxS), so that a row's
// result does not depend on how many activation rows share the call.
int gemv_plan_fixed(GemvArgs& a, int dev, int* grid_out, size_t* smem_out) {
    if (a.kparts <= 0) {
        GemvArgs probe = a;
        probe.S = kMaxS;
        int g;
        size_t sm;
        int rc = gemv_plan(probe, dev, &g, &sm);
        if (rc) return rc;
        a.kparts = probe.kparts;
    }
    return gemv_plan(a, dev, grid_out, smem_out);
}

int run_gemv(int epi, const GemvArgs& base, int dev, cudaStream_t st, bool pdl) {
    GemvArgs a = base;
    int grid;
    size_t smem;
    int rc = gemv_plan(a, dev, &grid, &smem);
    if (rc) return rc;
    cudaError_t e = launch_gemv(epi, a, grid, smem, st, pdl);
    if (e != cudaSuccess) return cuda_fail(e, "matvec launch");
    return SD_OK;
}

// Grow-only per-device workspace for partial outputs of K-split single-op matvecs.
float* op_workspace(int dev, size_t floats) {
    static float* ws[64] = {nullptr};
    static size_t cap[64] = {0};
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64) return nullptr;
    if (cap[dev] < floats) {
        cudaFree(ws[dev]);
        ws[dev] = nullptr;
        cap[dev] = 0;
        if (cudaMalloc(&ws[dev], floats * sizeof(float)) != cudaSuccess) return nullptr;
        cap[dev] = floats;
    }
    return ws[dev];
}

}  // namespace sd

// =============================================================================================
extern "C" {

const char* sd_last_error(void) { return sd::g_err.c_str(); }
int sd_abi_version(void) { return SD_ABI_VERSION; }

int sd_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int sd_qmat_create(const void* q4_0_host, int rows, int cols, int device, sd_qmat** out) {
    clear_error();
    if (!q4_0_host || !out || rows <= 0 || cols <= 0) return fail(SD_ERR_INVALID, "sd_qmat_create: bad arguments");
    if (cols % 1024 != 0) return fail(SD_ERR_INVALID, "sd_qmat_create: cols %d not a multiple of 1024", cols);
    if (sd_device_count() == 0) return fail(SD_ERR_NO_DEVICE, "no CUDA device");
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    const size_t aos_bytes = (size_t)rows * (cols / 32) * 18;
    const size_t bytes = qmat_bytes(rows, cols);
    uint8_t *tmp = nullptr, *w = nullptr;
    if ((e = cudaMalloc(&tmp, aos_bytes)) != cudaSuccess) return cuda_fail(e, "cudaMalloc");
    if ((e = cudaMalloc(&w, bytes)) != cudaSuccess) {
        cudaFree(tmp);
        return cuda_fail(e, "cudaMalloc");
    }
    int rc = SD_OK;
    if ((e = cudaMemcpy(tmp, q4_0_host, aos_bytes, cudaMemcpyHostToDevice)) != cudaSuccess) rc = cuda_fail(e, "upload");
    if (rc == SD_OK && (e = cudaMemset(w, 0, bytes)) != cudaSuccess) rc = cuda_fail(e, "memset");
    if (rc == SD_OK) rc = repack_matrix(tmp, rows, cols, RowMap{rows, 0, 0}, w, 0);
    if (rc == SD_OK && (e = cudaDeviceSynchronize()) != cudaSuccess) rc = cuda_fail(e, "repack");
    cudaFree(tmp);
    if (rc != SD_OK) {
        cudaFree(w);
        return rc;
    }
    sd_qmat* m = new sd_qmat{rows, cols, device, w, bytes};
    *out = m;
    return SD_OK;
}

void sd_qmat_free(sd_qmat* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    cudaFree(m->w);
    delete m;
}

int sd_qmat_shape(const sd_qmat* m, int* rows, int* cols, size_t* device_bytes) {
    if (!m) return fail(SD_ERR_INVALID, "null matrix");
    if (rows) *rows = m->rows;
    if (cols) *cols = m->cols;
    if (device_bytes) *device_bytes = m->bytes;
    return SD_OK;
}

int sd_quantize_q8_0_dev(const float* x, sd_q8_dev out, int S, int n, void* stream) {
    clear_error();
    if (!x || !out.qs || !out.d || !out.sum || S <= 0 || n <= 0 || n % 32)
        return fail(SD_ERR_INVALID, "sd_quantize_q8_0_dev: bad arguments");
    cudaError_t e = launch_quantize(x, Q8Planes{out.qs, out.d, out.sum}, S, n, (cudaStream_t)stream);
    return e == cudaSuccess ? SD_OK : cuda_fail(e, "quantize");
}

int sd_q8_to_blocks_dev(sd_q8_dev in, sd_block_q8_0* out, int S, int n, void* stream) {
    clear_error();
    if (!out || !in.qs || !in.d || S <= 0 || n <= 0 || n % 32) return fail(SD_ERR_INVALID, "bad arguments");
    cudaError_t e = launch_q8_to_blocks(Q8Planes{in.qs, in.d, in.sum}, out, S, n, (cudaStream_t)stream);
    return e == cudaSuccess ? SD_OK : cuda_fail(e, "q8_to_blocks");
}

int sd_blocks_to_q8_dev(const sd_block_q8_0* in, sd_q8_dev out, int S, int n, void* stream) {
    clear_error();
    if (!in || !out.qs || !out.d || !out.sum || S <= 0 || n <= 0 || n % 32) return fail(SD_ERR_INVALID, "bad arguments");
    cudaError_t e = launch_blocks_to_q8(in, Q8Planes{out.qs, out.d, out.sum}, S, n, (cudaStream_t)stream);
    return e == cudaSuccess ? SD_OK : cuda_fail(e, "blocks_to_q8");
}

static int matvec_common(int epi, const sd_qmat* W, sd_q8_dev x, float* y, int32_t* isum, int S, void* stream) {
    if (!W || !x.qs || !x.d || !x.sum) return fail(SD_ERR_INVALID, "matvec: null argument");
    int dev = W->device;
    int prc = check_current_device(dev, "matvec");
    if (prc) return prc;
    if ((prc = gemv_prepare_device(dev))) return prc;
    cudaStream_t st = (cudaStream_t)stream;
    GemvArgs a = {};
    a.w = W->w;
    a.n_rg = qmat_row_groups(W->rows);
    a.nq = W->cols / 128;
    a.K = W->cols;
    a.rg_per_unit = kRPW;
    a.n_units = a.n_rg / kRPW;
    a.act = Q8Planes{x.qs, x.d, x.sum};
    a.S = S;
    a.ctrl = nullptr;
    a.err = device_error_word(dev);
    a.out_ld = W->rows;
    a.out_rows = W->rows;
    a.isum = isum;
    a.kparts = 0;
    int grid;
    size_t smem;
    int rc = gemv_plan_fixed(a, dev, &grid, &smem);
    if (rc) return rc;
    const size_t n_out = (size_t)S * W->rows;
    float* parts = nullptr;
    if (epi == EPI_STORE) {
        if (a.kparts > 1) {
            parts = op_workspace(dev, n_out * a.kparts);
            if (!parts) return fail(SD_ERR_OOM, "matvec workspace");
            a.out = parts;
            a.part_stride = n_out;
        } else {
            a.out = y;
        }
    }
    // Programmatic dependent launch: the producer streams the matrix (written once, at sd_qmat_create) while the
    // stream's previous kernel drains; the kernel waits for that kernel before it reads x or writes y.
    cudaError_t e = launch_gemv(epi, a, grid, smem, st, true);
    if (e == cudaSuccess && parts) e = launch_sum_parts(parts, y, (int)n_out, a.kparts, n_out, st);
    return e == cudaSuccess ? SD_OK : cuda_fail(e, "matvec launch");
}

int sd_matvec_q4_0_q8_0_dev(const sd_qmat* W, sd_q8_dev x, float* y, int S, void* stream) {
    clear_error();
    if (!y) return fail(SD_ERR_INVALID, "matvec: null y");
    return matvec_common(EPI_STORE, W, x, y, nullptr, S, stream);
}

int sd_block_sums_dev(const sd_qmat* W, sd_q8_dev x, int32_t* isum, void* stream) {
    clear_error();
    if (!isum) return fail(SD_ERR_INVALID, "block sums: null output");
    if (W && W->rows % kTileRows) return fail(SD_ERR_INVALID, "block sums: rows %% 16 != 0");
    return matvec_common(EPI_BLOCKSUMS, W, x, nullptr, isum, 1, stream);
}

// ------------------------------- host-pointer drop-ins ---------------------------------------
namespace {
struct HostScratch {
    int dev = -1;
    size_t cap_x = 0, cap_y = 0, cap_blk = 0;
    float* x = nullptr;
    float* y = nullptr;
    uint8_t* blk = nullptr;
    int8_t* qs = nullptr;
    float* d = nullptr;
    int32_t* sum = nullptr;
    cudaStream_t st = nullptr;
};
std::mutex g_host_mu;
HostScratch g_hs;
std::map<std::tuple<const void*, int, int, int>, sd_qmat*> g_wcache;

int host_prepare(int n_in, int n_out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    HostScratch& h = g_hs;
    if (h.dev != dev) {
        cudaFree(h.x); cudaFree(h.y); cudaFree(h.blk); cudaFree(h.qs); cudaFree(h.d); cudaFree(h.sum);
        if (h.st) cudaStreamDestroy(h.st);
        h = HostScratch();
        h.dev = dev;
        if ((e = cudaStreamCreateWithFlags(&h.st, cudaStreamNonBlocking)) != cudaSuccess) return cuda_fail(e, "stream");
    }
    size_t need_x = (size_t)n_in, need_y = (size_t)n_out;
    if (need_x > h.cap_x) {
        cudaFree(h.x); cudaFree(h.blk); cudaFree(h.qs); cudaFree(h.d); cudaFree(h.sum);
        h.x = nullptr; h.blk = nullptr; h.qs = nullptr; h.d = nullptr; h.sum = nullptr;
        if ((e = cudaMalloc(&h.x, need_x * 4)) != cudaSuccess ||
            (e = cudaMalloc(&h.blk, need_x / 32 * 36)) != cudaSuccess ||
            (e = cudaMalloc(&h.qs, need_x)) != cudaSuccess || (e = cudaMalloc(&h.d, need_x / 32 * 4)) != cudaSuccess ||
            (e = cudaMalloc(&h.sum, need_x / 32 * 4)) != cudaSuccess) {
            h.cap_x = 0;
            return cuda_fail(e, "cudaMalloc");
        }
        h.cap_x = need_x;
    }
    if (need_y > h.cap_y) {
        cudaFree(h.y);
        h.y = nullptr;
        if ((e = cudaMalloc(&h.y, need_y * 4)) != cudaSuccess) {
            h.cap_y = 0;
            return cuda_fail(e, "cudaMalloc");
        }
        h.cap_y = need_y;
    }
    return SD_OK;
}
}  // namespace

void sd_host_quantize_f32_to_q8_0(const float* x, sd_block_q8_0* out, int n) {
    std::lock_guard<std::mutex> lk(g_host_mu);
    clear_error();
    int rc = (x && out && n > 0 && n % 32 == 0) ? host_prepare(n, 0) : fail(SD_ERR_INVALID, "quantize: bad arguments");
    HostScratch& h = g_hs;
    cudaError_t e = cudaSuccess;
    if (rc == SD_OK) {
        e = cudaMemcpyAsync(h.x, x, (size_t)n * 4, cudaMemcpyHostToDevice, h.st);
        if (e == cudaSuccess) e = launch_quantize(h.x, Q8Planes{h.qs, h.d, h.sum}, 1, n, h.st);
        if (e == cudaSuccess) e = launch_q8_to_blocks(Q8Planes{h.qs, h.d, h.sum}, h.blk, 1, n, h.st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(out, h.blk, (size_t)n / 32 * 36, cudaMemcpyDeviceToHost, h.st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(h.st);
        if (e != cudaSuccess) rc = cuda_fail(e, "quantize_f32_to_q8_0");
    }
    if (rc != SD_OK) fprintf(stderr, "specdec_b200: %s\n", sd_last_error());
}

void sd_host_q4_0_q8_0_matvec(const void* W, const sd_block_q8_0* x, float* y, int out_dim, int in_dim) {
    std::lock_guard<std::mutex> lk(g_host_mu);
    clear_error();
    int rc = (W && x && y && out_dim > 0 && in_dim > 0) ? host_prepare(in_dim, out_dim)
                                                         : fail(SD_ERR_INVALID, "matvec: bad arguments");
    HostScratch& h = g_hs;
    sd_qmat* m = nullptr;
    if (rc == SD_OK) {
        auto key = std::make_tuple(W, out_dim, in_dim, h.dev);
        auto it = g_wcache.find(key);
        if (it != g_wcache.end()) {
            m = it->second;
        } else {
            rc = sd_qmat_create(W, out_dim, in_dim, h.dev, &m);
            if (rc == SD_OK) g_wcache[key] = m;
        }
    }
    if (rc == SD_OK) {
        cudaError_t e = cudaMemcpyAsync(h.blk, x, (size_t)in_dim / 32 * 36, cudaMemcpyHostToDevice, h.st);
        if (e == cudaSuccess) e = launch_blocks_to_q8(h.blk, Q8Planes{h.qs, h.d, h.sum}, 1, in_dim, h.st);
        if (e != cudaSuccess) rc = cuda_fail(e, "matvec upload");
    }
    if (rc == SD_OK) rc = matvec_common(EPI_STORE, m, sd_q8_dev{h.qs, h.d, h.sum}, h.y, nullptr, 1, h.st);
    if (rc == SD_OK) {
        cudaError_t e = cudaMemcpyAsync(y, h.y, (size_t)out_dim * 4, cudaMemcpyDeviceToHost, h.st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(h.st);
        if (e != cudaSuccess) rc = cuda_fail(e, "matvec download");
    }
    if (rc == SD_OK) rc = check_device_error(device_error_word(h.dev), h.st);
    if (rc != SD_OK) fprintf(stderr, "specdec_b200: %s\n", sd_last_error());
}

int sd_device_error(int device) {
    clear_error();
    int* w = device_error_word(device);
    if (!w) return fail(SD_ERR_INVALID, "sd_device_error: no error word on device %d", device);
    int h = 0;
    cudaError_t e = cudaMemcpy(&h, w, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
    if (h != 0 && (e = cudaMemset(w, 0, sizeof(int))) != cudaSuccess) return cuda_fail(e, "clearing the device error word");
    return h;
}

void sd_host_kq_matvec(int type, const void* W, const float* x, float* y, int out_dim, int in_dim) {
    std::lock_guard<std::mutex> lk(g_host_mu);
    clear_error();
    int rc = (W && x && y && out_dim > 0 && in_dim > 0 && in_dim % 256 == 0 && (type == kTypeQ6K || type == kTypeQ4K))
                 ? host_prepare(in_dim, out_dim)
                 : fail(SD_ERR_INVALID, "kq matvec: bad arguments (type 12 or 14, in_dim %% 256 == 0)");
    HostScratch& h = g_hs;
    uint8_t* wd = nullptr;
    if (rc == SD_OK) {
        // the device copy of W (the layout of sd_kquant.h), cached per (address, type, shape, device) like the Q4_0 one
        static std::map<std::tuple<const void*, int, int, int, int>, uint8_t*> cache;
        auto key = std::make_tuple(W, type, out_dim, in_dim, h.dev);
        auto it = cache.find(key);
        if (it != cache.end()) {
            wd = it->second;
        } else {
            const size_t n_blocks = (size_t)out_dim * (in_dim / 256);
            const size_t raw = n_blocks * (type == kTypeQ6K ? kQ6KBytes : kQ4KBytes);
            cudaError_t e = cudaMalloc(&wd, (size_t)out_dim * kq_device_row_bytes(type, in_dim));
            if (e == cudaSuccess && type == kTypeQ4K) {
                e = cudaMemcpy(wd, W, raw, cudaMemcpyHostToDevice);
            } else if (e == cudaSuccess) {
                uint8_t* tmp = nullptr;
                e = cudaMalloc(&tmp, raw);
                if (e == cudaSuccess) e = cudaMemcpy(tmp, W, raw, cudaMemcpyHostToDevice);
                if (e == cudaSuccess) e = launch_repack_q6k(tmp, wd, n_blocks, h.st);
                if (e == cudaSuccess) e = cudaStreamSynchronize(h.st);
                cudaFree(tmp);
            }
            if (e != cudaSuccess) {
                cudaFree(wd);
                wd = nullptr;
                rc = cuda_fail(e, "kq matvec upload");
            } else {
                cache[key] = wd;
            }
        }
    }
    if (rc == SD_OK) {
        cudaError_t e = cudaMemcpyAsync(h.x, x, (size_t)in_dim * 4, cudaMemcpyHostToDevice, h.st);
        if (e == cudaSuccess) e = launch_kq_matvec(type, wd, out_dim, in_dim, h.x, h.y, out_dim, 1, nullptr, h.st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(y, h.y, (size_t)out_dim * 4, cudaMemcpyDeviceToHost, h.st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(h.st);
        if (e != cudaSuccess) rc = cuda_fail(e, "kq matvec");
    }
    if (rc != SD_OK) fprintf(stderr, "specdec_b200: %s\n", sd_last_error());
}

void sd_host_cache_clear(void) {
    std::lock_guard<std::mutex> lk(g_host_mu);
    for (auto& kv : g_wcache) sd_qmat_free(kv.second);
    g_wcache.clear();
}

}  // extern "C"

// ------------------------------- allocation-free matvec --------------------------------------
// Some callers cannot let a library allocate device memory at call time: a serving process that
// hands all free HBM to its own pool at start-up (a late cudaMalloc fails there), or a latency loop
// that cannot take the device-wide synchronisation of the cudaFree that sd_matvec_q4_0_q8_0_dev
// performs when its partial-output workspace grows.  For them the K-split partial outputs live in a
// fixed array below, which every GPU that loads this library holds until the process exits.
namespace sd {

static __device__ __align__(256) float g_noalloc_parts[SD_NOALLOC_SCRATCH_BYTES / sizeof(float)];

// Device address of g_noalloc_parts on `dev`, looked up once per device with that device current.
// In host code the name g_noalloc_parts is only a host-side stand-in; kernels get this address.
static int noalloc_scratch(int dev, float** out) {
    static float* addr[64] = {nullptr};
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64) return fail(SD_ERR_INVALID, "no-alloc matvec: bad device %d", dev);
    if (!addr[dev]) {
        int prev = -1;
        cudaError_t e = cudaGetDevice(&prev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
        if (prev != dev && (e = cudaSetDevice(dev)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
        float* p = nullptr;
        e = cudaGetSymbolAddress((void**)&p, g_noalloc_parts);
        if (prev != dev) cudaSetDevice(prev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress (no-alloc matvec scratch)");
        addr[dev] = p;
    }
    *out = addr[dev];
    return SD_OK;
}

}  // namespace sd

extern "C" int sd_matvec_q4_0_q8_0_noalloc_dev(const sd_qmat* W, sd_q8_dev x, float* y, int S, void* stream) {
    clear_error();
    if (!W || !x.qs || !x.d || !x.sum || !y) return fail(SD_ERR_INVALID, "no-alloc matvec: null argument");
    const int dev = W->device;
    int rc = check_current_device(dev, "no-alloc matvec");
    if (rc) return rc;
    if ((rc = gemv_prepare_device(dev))) return rc;
    float* scratch = nullptr;
    if ((rc = noalloc_scratch(dev, &scratch))) return rc;
    GemvArgs a = {};
    a.w = W->w;
    a.n_rg = qmat_row_groups(W->rows);
    a.nq = W->cols / 128;
    a.K = W->cols;
    a.rg_per_unit = kRPW;
    a.n_units = a.n_rg / kRPW;
    a.act = Q8Planes{x.qs, x.d, x.sum};
    a.S = S;
    a.ctrl = nullptr;
    a.err = device_error_word(dev);  // a file-scope device variable: no allocation (sd_device_error reads it)
    a.out_ld = W->rows;
    a.out_rows = W->rows;
    a.kparts = 0;
    int grid;
    size_t smem;
    if ((rc = gemv_plan_fixed(a, dev, &grid, &smem))) return rc;
    const size_t n_out = (size_t)S * W->rows;
    const cudaStream_t st = (cudaStream_t)stream;
    if (a.kparts > 1) {
        const size_t need = n_out * a.kparts * sizeof(float);
        if (need > SD_NOALLOC_SCRATCH_BYTES)
            return fail(SD_ERR_INVALID,
                        "no-alloc matvec: %d x %d at S=%d splits K into %d parts and needs %zu bytes of scratch; "
                        "the limit is %zu bytes (use sd_matvec_q4_0_q8_0_dev)",
                        W->rows, W->cols, S, a.kparts, need, (size_t)SD_NOALLOC_SCRATCH_BYTES);
        // Every partial that k_sum_parts reads is written by this call's matvec first, so the array
        // needs no clearing between calls.
        a.out = scratch;
        a.part_stride = n_out;
    } else {
        a.out = y;
    }
    cudaError_t e = launch_gemv(EPI_STORE, a, grid, smem, st, false);
    if (e == cudaSuccess && a.kparts > 1) e = launch_sum_parts(scratch, y, (int)n_out, a.kparts, n_out, st);
    return e == cudaSuccess ? SD_OK : cuda_fail(e, "no-alloc matvec launch");
}
