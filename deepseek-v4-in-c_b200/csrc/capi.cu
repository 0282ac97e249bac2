// capi.cu - the reference-compatible C ABI (include/dsv4_b200.h, layer 1) and
// the device GEMV entry (layer 2).
//
// Mirrors include/dsv4/dsv4_cuda.h of the reference: same symbols, same 0/-1
// contract, abort() on misuse (src/cuda/dsv4_cuda.cu:387-434). Differences by
// design: weights of every format can be resident, residency resolves row
// slices of a resident matrix, and host<->device traffic goes through pinned
// staging on one non-blocking stream with a single synchronisation per call.
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "moe.h"
#include "../../include/dsv4_b200.h"

namespace dsv4b {

struct Resident {
    const void *key;        // host m->w
    const void *skey;       // host m->s
    uint8_t *dw, *ds;       // device copies
    int wdt, rows, cols, blk_r, blk_c, sc;
    size_t wbytes, sbytes, rowbytes;
    bool f16s;              // FP4: every scale f16-safe (checked at upload)
};

struct State {
    int ready = 0, dev = 0;
    cudaStream_t st = nullptr;
    std::vector<Resident> res;
    float *dx = nullptr, *dy = nullptr, *hx = nullptr, *hy = nullptr;
    size_t xcap = 0, ycap = 0, hxcap = 0, hycap = 0;
};
State g;

cudaStream_t stream_of(void *s) { return s ? (cudaStream_t)s : g.st; }

int smem_optin(const void *kernel, int bytes)
{
    static std::mutex mu;
    static std::vector<std::pair<int, const void *>> done;   // (device, kernel) pairs already raised
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    std::lock_guard<std::mutex> lk(mu);
    for (const auto &d : done)
        if (d.first == dev && d.second == kernel) return 0;
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) {
        fprintf(stderr, "dsv4_b200: raising a kernel's shared memory to %d bytes on device %d failed: %s\n", bytes,
                dev, cudaGetErrorString(e));
        return -1;
    }
    done.emplace_back(dev, kernel);
    return 0;
}

thread_local int t_chain = 0;
thread_local bool t_pdl = false;

bool pdl_enabled()
{
    static const bool on = [] {
        const char *e = getenv("DSV4B_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

static int scale_rows(int rows, int blk_r) { return (rows + blk_r - 1) / blk_r; }

// Exact residency, then containment: a matrix whose host rows are whole
// row-blocks inside a resident matrix of the same format and width is that
// matrix's slice (the grouped wo_a call, dsv4_layer.c:321-334). `row0` is the
// first row of the slice within the resident matrix.
static const Resident *find(const DSV4QMat *m, int *row0)
{
    if (!m || !m->w) return nullptr;
    for (const Resident &r : g.res)
        if (r.key == m->w && r.rows == m->rows && r.cols == m->cols && r.wdt == m->wdt) {
            *row0 = 0;
            return &r;
        }
    for (const Resident &r : g.res) {
        if (r.wdt != m->wdt || r.cols != m->cols) continue;
        const uint8_t *base = (const uint8_t *)r.key, *p = (const uint8_t *)m->w;
        if (p < base || p >= base + r.wbytes) continue;
        const size_t off = (size_t)(p - base);
        if (off % r.rowbytes) continue;
        const int o0 = (int)(off / r.rowbytes);
        if (o0 + m->rows > r.rows) continue;
        if (r.wdt >= DSV4_WFP8) {
            if (o0 % r.blk_r || m->blk_r != r.blk_r || m->blk_c != r.blk_c) continue;
            const uint8_t *sp = (const uint8_t *)r.skey + (size_t)(o0 / r.blk_r) * r.sc;
            if ((const uint8_t *)m->s != sp) continue;
        }
        *row0 = o0;
        return &r;
    }
    return nullptr;
}

static int stage(size_t xn, size_t yn)
{
    if (xn > g.xcap) {
        if (g.dx) cudaFree(g.dx);
        g.dx = nullptr; g.xcap = 0;
        DSV4B_CUDA_OK(cudaMalloc(&g.dx, xn * sizeof(float)));
        g.xcap = xn;
    }
    if (yn > g.ycap) {
        if (g.dy) cudaFree(g.dy);
        g.dy = nullptr; g.ycap = 0;
        DSV4B_CUDA_OK(cudaMalloc(&g.dy, yn * sizeof(float)));
        g.ycap = yn;
    }
    if (xn > g.hxcap) {
        if (g.hx) cudaFreeHost(g.hx);
        g.hx = nullptr; g.hxcap = 0;
        DSV4B_CUDA_OK(cudaHostAlloc(&g.hx, xn * sizeof(float), cudaHostAllocDefault));
        g.hxcap = xn;
    }
    if (yn > g.hycap) {
        if (g.hy) cudaFreeHost(g.hy);
        g.hy = nullptr; g.hycap = 0;
        DSV4B_CUDA_OK(cudaHostAlloc(&g.hy, yn * sizeof(float), cudaHostAllocDefault));
        g.hycap = yn;
    }
    return 0;
}

// Host-buffer GEMV through pinned staging: one H2D, the kernel, one D2H, one
// stream synchronisation.
static int host_gemv(float *y, const float *x, const Resident &r, int row0, int rows, int nt)
{
    const size_t xn = (size_t)nt * r.cols, yn = (size_t)nt * rows;
    if (stage(xn, yn) != 0) return -1;
    memcpy(g.hx, x, xn * sizeof(float));
    DSV4B_CUDA_OK(cudaMemcpyAsync(g.dx, g.hx, xn * sizeof(float), cudaMemcpyHostToDevice, g.st));
    const uint8_t *dw = r.dw + (size_t)row0 * r.rowbytes;
    const uint8_t *ds = r.ds ? r.ds + (size_t)(row0 / r.blk_r) * r.sc : nullptr;
    if (gemv(r.wdt, g.dy, rows, g.dx, r.cols, dw, ds, rows, r.cols, r.blk_r, r.blk_c, nt, g.st, r.f16s) != 0)
        return -1;
    DSV4B_CUDA_OK(cudaMemcpyAsync(g.hy, g.dy, yn * sizeof(float), cudaMemcpyDeviceToHost, g.st));
    DSV4B_CUDA_OK(cudaStreamSynchronize(g.st));
    memcpy(y, g.hy, yn * sizeof(float));
    return 0;
}

}  // namespace dsv4b

using namespace dsv4b;

extern "C" int dsv4_cuda_available(void)
{
    int n = 0;
    return (cudaGetDeviceCount(&n) == cudaSuccess && n > 0) ? 1 : 0;
}

extern "C" int dsv4_cuda_set_blocking_sync(void)
{
    DSV4B_CUDA_OK(cudaSetDeviceFlags(cudaDeviceScheduleBlockingSync));
    return 0;
}

extern "C" int dsv4_cuda_init(void)
{
    if (g.ready) return 0;
    int n = 0;
    DSV4B_CUDA_OK(cudaGetDeviceCount(&n));
    if (n < 1) { fprintf(stderr, "dsv4_b200: no device\n"); return -1; }
    const char *e = getenv("DSV4_DEVICE");
    g.dev = e ? atoi(e) : 0;
    if (g.dev < 0 || g.dev >= n) { fprintf(stderr, "dsv4_b200: DSV4_DEVICE=%d of %d\n", g.dev, n); return -1; }
    DSV4B_CUDA_OK(cudaSetDevice(g.dev));
    cudaDeviceProp p;
    DSV4B_CUDA_OK(cudaGetDeviceProperties(&p, g.dev));
    if (p.major != 10) {
        fprintf(stderr, "dsv4_b200: built for sm_100a, device is sm_%d%d\n", p.major, p.minor);
        return -1;
    }
    DSV4B_CUDA_OK(cudaStreamCreateWithFlags(&g.st, cudaStreamNonBlocking));
    size_t fr = 0, tot = 0;
    DSV4B_CUDA_OK(cudaMemGetInfo(&fr, &tot));
    printf("cuda: %s, sm_%d%d, %d SMs, %.2f GB free of %.2f GB\n", p.name, p.major, p.minor,
           p.multiProcessorCount, fr / 1073741824.0, tot / 1073741824.0);
    g.ready = 1;
    return 0;
}

extern "C" size_t dsv4_cuda_free_vram(void)
{
    size_t fr = 0, tot = 0;
    if (!g.ready || cudaMemGetInfo(&fr, &tot) != cudaSuccess) return 0;
    return fr;
}

extern "C" int dsv4_cuda_has(const DSV4QMat *m)
{
    int row0;
    return (g.ready && find(m, &row0)) ? 1 : 0;
}

extern "C" int dsv4_cuda_upload(const DSV4QMat *m)
{
    if (!g.ready || !m || !m->w || m->rows <= 0 || m->cols <= 0) return -1;
    if (m->wdt < DSV4_WF32 || m->wdt > DSV4_WFP4) return -1;
    const bool scaled = m->wdt >= DSV4_WFP8;
    if (scaled && (!m->s || m->blk_r <= 0 || m->blk_c <= 0)) return -1;
    if (m->wdt == DSV4_WFP4 && (m->cols & 1)) return -1;
    int row0;
    const Resident *have = find(m, &row0);
    if (have && row0 == 0 && have->key == m->w) return 0;

    Resident r = {};
    r.key = m->w; r.skey = m->s; r.wdt = m->wdt;
    r.rows = m->rows; r.cols = m->cols;
    r.blk_r = scaled ? m->blk_r : 1; r.blk_c = scaled ? m->blk_c : 1;
    r.sc = scaled ? (m->cols + m->blk_c - 1) / m->blk_c : 0;
    r.rowbytes = row_bytes(m->wdt, m->cols);
    r.wbytes = r.rowbytes * (size_t)m->rows;
    r.sbytes = scaled ? (size_t)scale_rows(m->rows, m->blk_r) * r.sc : 0;
    r.f16s = m->wdt == DSV4_WFP4 && scaled && fp4_scales_f16((const uint8_t *)m->s, r.sbytes);
    // Headroom, as the reference keeps (dsv4_cuda.cu:317-320).
    if (r.wbytes + r.sbytes + (256u << 20) > dsv4_cuda_free_vram()) return -1;
    if (cudaMalloc(&r.dw, r.wbytes) != cudaSuccess) return -1;
    if (r.sbytes && cudaMalloc(&r.ds, r.sbytes) != cudaSuccess) { cudaFree(r.dw); return -1; }
    if (cudaMemcpy(r.dw, m->w, r.wbytes, cudaMemcpyHostToDevice) != cudaSuccess ||
        (r.sbytes && cudaMemcpy(r.ds, m->s, r.sbytes, cudaMemcpyHostToDevice) != cudaSuccess)) {
        cudaFree(r.dw);
        if (r.ds) cudaFree(r.ds);
        return -1;
    }
    g.res.push_back(r);
    return 0;
}

extern "C" int dsv4_cuda_evict(const DSV4QMat *m)
{
    if (!g.ready || !m) return -1;
    for (size_t i = 0; i < g.res.size(); i++) {
        Resident &r = g.res[i];
        if (r.key == m->w && r.rows == m->rows && r.cols == m->cols && r.wdt == m->wdt) {
            cudaStreamSynchronize(g.st);
            cudaFree(r.dw);
            if (r.ds) cudaFree(r.ds);
            g.res.erase(g.res.begin() + (long)i);
            return 0;
        }
    }
    return -1;
}

extern "C" int dsv4_cuda_resident_ptrs(const DSV4QMat *m, const void **dw, const void **ds)
{
    int row0;
    const Resident *r = g.ready ? find(m, &row0) : nullptr;
    if (!r) return -1;
    if (dw) *dw = r->dw + (size_t)row0 * r->rowbytes;
    if (ds) *ds = r->ds ? r->ds + (size_t)(row0 / r->blk_r) * r->sc : nullptr;
    return 0;
}

extern "C" void dsv4_cuda_mmq(float *y, const float *x, const DSV4QMat *m)
{
    int row0 = 0;
    const Resident *r = g.ready ? find(m, &row0) : nullptr;
    if (!r || host_gemv(y, x, *r, row0, m->rows, 1) != 0) {
        fprintf(stderr, "dsv4_b200: mmq called for a matrix that is not resident\n");
        abort();
    }
}

extern "C" void dsv4_cuda_mmq_n(float *y, const float *x, const DSV4QMat *m, int nt)
{
    if (nt <= 1) { dsv4_cuda_mmq(y, x, m); return; }
    int row0 = 0;
    const Resident *r = g.ready ? find(m, &row0) : nullptr;
    if (!r || nt > DSV4_MAX_BATCH || host_gemv(y, x, *r, row0, m->rows, nt) != 0) {
        fprintf(stderr, "dsv4_b200: mmq_n called for a matrix that is not resident, "
                        "or a batch that will not stage\n");
        abort();
    }
}

extern "C" void dsv4_cuda_shutdown(void)
{
    if (!g.ready) return;
    cudaStreamSynchronize(g.st);
    for (Resident &r : g.res) {
        cudaFree(r.dw);
        if (r.ds) cudaFree(r.ds);
    }
    g.res.clear();
    if (g.dx) cudaFree(g.dx);
    if (g.dy) cudaFree(g.dy);
    if (g.hx) cudaFreeHost(g.hx);
    if (g.hy) cudaFreeHost(g.hy);
    g.dx = g.dy = g.hx = g.hy = nullptr;
    g.xcap = g.ycap = g.hxcap = g.hycap = 0;
    cudaStreamDestroy(g.st);
    g.st = nullptr;
    g.ready = 0;
}

extern "C" int dsv4_cuda_dump_e4m3(float *host256)
{
    if (!g.ready && dsv4_cuda_init() != 0) return -1;
    float *d = nullptr;
    DSV4B_CUDA_OK(cudaMalloc(&d, 256 * sizeof(float)));
    int rc = dump_e4m3(d, g.st);
    if (rc == 0 && cudaMemcpyAsync(host256, d, 256 * sizeof(float), cudaMemcpyDeviceToHost, g.st) != cudaSuccess) rc = -1;
    if (cudaStreamSynchronize(g.st) != cudaSuccess) rc = -1;
    cudaFree(d);
    return rc;
}

extern "C" int dsv4b_gemv(int wdt, float *y, const float *x, const void *W, const void *S,
                          int rows, int cols, int blk_r, int blk_c, int nt, void *stream)
{
    if (wdt < DSV4_WF32 || wdt > DSV4_WFP4 || !y || !x || !W) return -1;
    if (wdt >= DSV4_WFP8 && (!S || blk_r <= 0 || blk_c <= 0)) return -1;
    return gemv(wdt, y, rows, x, cols, W, (const uint8_t *)S, rows, cols, blk_r, blk_c, nt,
                stream_of(stream));
}

// ------------------------------------------------------------------- MoE ---

namespace dsv4b {

static bool devmat(const DSV4QMat *m, DevMat &d)
{
    int row0 = 0;
    const Resident *r = find(m, &row0);
    if (!r) return false;
    d.w = r->dw + (size_t)row0 * r->rowbytes;
    d.s = r->ds ? r->ds + (size_t)(row0 / r->blk_r) * r->sc : nullptr;
    d.wdt = r->wdt;
    d.rows = m->rows;
    d.cols = m->cols;
    d.blk_r = r->blk_r;
    d.blk_c = r->blk_c;
    d.f16s = r->f16s ? 1 : 0;
    return true;
}

}  // namespace dsv4b

struct dsv4b_moe {
    dsv4b::MoeLayer L;
    dsv4b::MoeScratch S;
    void *tables;       // 6 x n_experts device pointers
    float *scratch;
    float *bias;
    int *fixed;
    float *dx, *dout;
};

extern "C" dsv4b_moe *dsv4_cuda_moe_prepare(const DSV4QMat *gate, const float *bias,
                                            const DSV4QMat *experts, int n_experts,
                                            const DSV4QMat *shared, int topk, float route_scale,
                                            int score_func, float swiglu_limit)
{
    using namespace dsv4b;
    if (!g.ready || !gate || !experts || n_experts < 1 || n_experts > kMoeMaxExperts || topk < 1 ||
        topk > kMoeMaxTopk || topk > n_experts || (score_func != 1 && score_func != 2))
        return nullptr;
    dsv4b_moe *m = (dsv4b_moe *)calloc(1, sizeof *m);
    if (!m) return nullptr;
    MoeLayer &L = m->L;
    bool ok = devmat(gate, L.gate);
    L.n_experts = n_experts;
    L.topk = topk;
    L.hidden = gate->cols;
    L.inter = experts[0].rows;
    L.efmt = experts[0].wdt;
    L.eblk_r = experts[0].blk_r;
    L.eblk_c = experts[0].blk_c;
    L.route_scale = route_scale;
    L.score_func = score_func;
    L.swiglu_limit = swiglu_limit;
    std::vector<const uint8_t *> tab((size_t)6 * n_experts, nullptr);
    L.ef16s = 1;
    for (int e = 0; ok && e < n_experts; e++) {
        const DSV4QMat *x3 = experts + 3 * e;
        for (int j = 0; j < 3 && ok; j++) {
            DevMat d;
            ok = devmat(&x3[j], d) && x3[j].wdt == L.efmt;
            if (!ok) break;
            const int want_rows = (j == 2) ? L.hidden : L.inter, want_cols = (j == 2) ? L.inter : L.hidden;
            ok = (d.rows == want_rows && d.cols == want_cols);
            tab[(size_t)(2 * j) * n_experts + e] = d.w;
            tab[(size_t)(2 * j + 1) * n_experts + e] = d.s;
            L.ef16s &= d.f16s;
        }
    }
    if (ok && shared) {
        L.has_shared = 1;
        for (int j = 0; j < 3 && ok; j++) ok = devmat(&shared[j], L.sh[j]);
        L.inter_shared = ok ? shared[0].rows : 0;
    }
    const size_t nf = moe_scratch_floats(L.hidden, L.inter, L.inter_shared, n_experts, topk);
    if (ok) ok = cudaMalloc(&m->tables, tab.size() * sizeof(void *)) == cudaSuccess &&
                 cudaMemcpy(m->tables, tab.data(), tab.size() * sizeof(void *), cudaMemcpyHostToDevice) == cudaSuccess;
    if (ok) ok = cudaMalloc(&m->scratch, (nf + kMoeMaxTopk) * sizeof(float)) == cudaSuccess;
    if (ok) ok = cudaMalloc(&m->fixed, kMoeMaxTopk * sizeof(int)) == cudaSuccess;
    if (ok) ok = cudaMalloc(&m->dx, (size_t)L.hidden * sizeof(float)) == cudaSuccess &&
                 cudaMalloc(&m->dout, (size_t)L.hidden * sizeof(float)) == cudaSuccess;
    if (ok && bias)
        ok = cudaMalloc(&m->bias, n_experts * sizeof(float)) == cudaSuccess &&
             cudaMemcpy(m->bias, bias, n_experts * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess;
    if (!ok) {
        dsv4_cuda_moe_free(m);
        return nullptr;
    }
    const uint8_t *const *t = (const uint8_t *const *)m->tables;
    L.w1tab = t; L.s1tab = t + n_experts;
    L.w3tab = t + 2 * n_experts; L.s3tab = t + 3 * n_experts;
    L.w2tab = t + 4 * n_experts; L.s2tab = t + 5 * n_experts;
    L.bias = m->bias;
    moe_scratch_carve(m->S, m->scratch, L.hidden, L.inter, L.inter_shared, n_experts, topk);
    return m;
}

extern "C" void dsv4_cuda_moe_free(dsv4b_moe *m)
{
    if (!m) return;
    if (g.st) cudaStreamSynchronize(g.st);
    cudaFree(m->tables);
    cudaFree(m->scratch);
    cudaFree(m->fixed);
    cudaFree(m->bias);
    cudaFree(m->dx);
    cudaFree(m->dout);
    free(m);
}

extern "C" int dsv4b_moe_forward(dsv4b_moe *m, float *out, const float *x, void *stream)
{
    if (!m) return -1;
    m->L.fixed = nullptr;
    return dsv4b::moe_forward(m->L, m->S, out, x, nullptr, stream_of(stream));
}

extern "C" int dsv4_cuda_moe(dsv4b_moe *m, float *out, const float *x, const int *fixed_experts,
                             int *idx_out, float *w_out)
{
    if (!m || !out || !x) return -1;
    const int H = m->L.hidden, K = m->L.topk;
    DSV4B_CUDA_OK(cudaMemcpyAsync(m->dx, x, (size_t)H * sizeof(float), cudaMemcpyHostToDevice, g.st));
    m->L.fixed = nullptr;
    if (fixed_experts) {
        for (int k = 0; k < K; k++)
            if (fixed_experts[k] < 0 || fixed_experts[k] >= m->L.n_experts) return -1;
        DSV4B_CUDA_OK(cudaMemcpyAsync(m->fixed, fixed_experts, K * sizeof(int), cudaMemcpyHostToDevice, g.st));
        m->L.fixed = m->fixed;
    }
    if (dsv4b::moe_forward(m->L, m->S, m->dout, m->dx, nullptr, g.st) != 0) return -1;
    DSV4B_CUDA_OK(cudaMemcpyAsync(out, m->dout, (size_t)H * sizeof(float), cudaMemcpyDeviceToHost, g.st));
    if (idx_out) DSV4B_CUDA_OK(cudaMemcpyAsync(idx_out, m->S.sel, K * sizeof(int), cudaMemcpyDeviceToHost, g.st));
    if (w_out) DSV4B_CUDA_OK(cudaMemcpyAsync(w_out, m->S.wts, K * sizeof(float), cudaMemcpyDeviceToHost, g.st));
    DSV4B_CUDA_OK(cudaStreamSynchronize(g.st));
    m->L.fixed = nullptr;
    return 0;
}
