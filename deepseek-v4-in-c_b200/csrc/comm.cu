// comm.cu - the multi-GPU exchange of a sharded decode step: NCCL over
// NVLink / NVSwitch, opened at run time (dlopen), so the single-GPU library
// has no NCCL dependency and a process that already loaded torch's NCCL
// shares that copy instead of loading a second one.
//
// Two exchanges are used: a sum all-reduce of f32 partials (the column-split
// wo_b output and the row-split experts' per-slot outputs) and an all-gather
// of each rank's LM-head argmax pair. All ranks enqueue the same collectives
// in the same order, in the eager first step and in the captured graph
// alike. The kernel launched after a collective depends on it fully (not as
// a programmatic dependent): a collective need not be a single kernel.
#include <dlfcn.h>
#include <nccl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "common.cuh"
#include "internal.h"

namespace dsv4b {

namespace {

struct Nccl {
    bool tried = false, ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    const char *(*error_string)(ncclResult_t);
} N;

template <typename F>
static bool sym(void *h, const char *name, F &f)
{
    f = reinterpret_cast<F>(dlsym(h, name));
    if (!f) fprintf(stderr, "dsv4_b200: NCCL symbol %s missing\n", name);
    return f != nullptr;
}

static bool nccl_load()
{
    if (N.tried) return N.ok;
    N.tried = true;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        fprintf(stderr, "dsv4_b200: cannot open NCCL (%s)\n", dlerror());
        return false;
    }
    N.ok = sym(h, "ncclGetUniqueId", N.get_unique_id) && sym(h, "ncclCommInitRank", N.comm_init_rank) &&
           sym(h, "ncclCommDestroy", N.comm_destroy) && sym(h, "ncclAllReduce", N.all_reduce) &&
           sym(h, "ncclAllGather", N.all_gather) && sym(h, "ncclGetErrorString", N.error_string);
    return N.ok;
}

static int check(ncclResult_t r, const char *what)
{
    if (r == ncclSuccess) return 0;
    fprintf(stderr, "dsv4_b200: %s failed: %s\n", what, N.error_string ? N.error_string(r) : "?");
    return -1;
}

}  // namespace

size_t comm_id_bytes() { return sizeof(ncclUniqueId); }

int comm_unique_id(void *out)
{
    if (!out || !nccl_load()) return -1;
    ncclUniqueId id;
    if (check(N.get_unique_id(&id), "ncclGetUniqueId")) return -1;
    memcpy(out, &id, sizeof id);
    return 0;
}

int comm_open(void **comm, int rank, int world, const void *id)
{
    *comm = nullptr;
    if (world < 2) return 0;
    if (!id || rank < 0 || rank >= world || !nccl_load()) return -1;
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof uid);
    ncclComm_t c = nullptr;
    if (check(N.comm_init_rank(&c, world, uid, rank), "ncclCommInitRank")) return -1;
    *comm = c;
    return 0;
}

void comm_close(void *comm)
{
    if (comm && N.ok) N.comm_destroy(static_cast<ncclComm_t>(comm));
}

int comm_allreduce_sum(float *buf, size_t n, void *comm, cudaStream_t st)
{
    if (!comm) return 0;
    t_pdl = false;
    return check(N.all_reduce(buf, buf, n, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), st),
                 "ncclAllReduce");
}

int comm_allgather(const void *send, void *recv, size_t bytes_per_rank, void *comm, cudaStream_t st)
{
    if (!comm) return 0;
    t_pdl = false;
    return check(N.all_gather(send, recv, bytes_per_rank, ncclUint8, static_cast<ncclComm_t>(comm), st),
                 "ncclAllGather");
}

}  // namespace dsv4b

// ------------------------------------------------- one-shot peer exchange
// A sum all-reduce of a small f32 vector over NVLink peer memory, in one
// kernel and without flags or fences: every rank owns a mailbox in its own
// HBM ([3 buffers][world][maxn] words), mapped into every other rank by CUDA
// IPC, whose empty words hold the sentinel -0.0 (0x80000000). An exchange
// stores this rank's values (a -0.0 sent as +0.0, the same number) into slot
// `rank` of buffer b of every mailbox; each thread then polls its words of
// its own mailbox (volatile loads, bounded) until no rank's word is the
// sentinel, sums them in rank order -- the same order on every rank, so all
// ranks get the same bits -- and re-arms the words with the sentinel. Aligned
// 4-byte stores arrive whole, so a word is either empty or final. The buffer
// of exchange x (x = step * exchanges per step + call, the step count kept on
// the device) is x mod 3: a rank writes buffer b again only after two more
// exchanges, which need every rank to have finished (and re-armed) this one.
namespace dsv4b {

namespace {

constexpr unsigned kSentinel = 0x80000000u;
constexpr unsigned kSpinLimit = 1u << 26;     // several seconds: a peer that never arrives

struct PeerDev {
    float *const *pmail;       // [world] every rank's mailbox
    float *mail;               // mine
    int *err;
    int rank, world, maxn;
    unsigned spin;             // polls before a wait gives up
};

// Polls before a wait for a rank gives up: kSpinLimit, or $DSV4B_PEER_SPIN.
unsigned peer_spin_limit()
{
    const char *e = getenv("DSV4B_PEER_SPIN");
    const long v = e ? atol(e) : 0;
    return v > 0 ? (unsigned)v : kSpinLimit;
}

struct PeerHost {
    PeerDev d;
    void *base;                // my mailbox
    void *misc;                // err, the pointer table
    std::vector<void *> opened;
};

__global__ void k_fill_u32(unsigned *p, size_t n, unsigned v)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) p[i] = v;
}

__device__ __forceinline__ uint4 ld_volatile_u4(const void *p)
{
    uint4 r;
    asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p) : "memory");
    return r;
}

__device__ __forceinline__ unsigned unsent(float v)
{
    const unsigned u = __float_as_uint(v);
    return u == kSentinel ? 0u : u;
}

__global__ void __launch_bounds__(256) k_peer_allreduce(PeerDev x, float *buf, int n, const unsigned *stepseq,
                                                        int nx, int call)
{
    pdl_trigger();
    pdl_wait();
    const int G = x.world, n4 = n >> 2;
    const unsigned xi = __ldcg(stepseq) * (unsigned)nx + (unsigned)call;
    const size_t slot = (size_t)x.maxn, bsz = (size_t)G * slot, b = xi % 3u;
    const int stride = gridDim.x * blockDim.x, i0 = blockIdx.x * blockDim.x + threadIdx.x;
    const float4 *b4 = reinterpret_cast<const float4 *>(buf);
    for (int i = i0; i < n4; i += stride) {
        const float4 v = __ldcg(b4 + i);
        const uint4 u = make_uint4(unsent(v.x), unsent(v.y), unsent(v.z), unsent(v.w));
        for (int r = 0; r < G; r++)
            reinterpret_cast<uint4 *>(x.pmail[r] + b * bsz + (size_t)x.rank * slot)[i] = u;
    }
    unsigned spins = 0;
    bool gave_up = false;
    for (int i = i0; i < n4; i += stride) {
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < G; r++) {
            uint4 *w = reinterpret_cast<uint4 *>(x.mail + b * bsz + (size_t)r * slot) + i;
            uint4 u = ld_volatile_u4(w);
            while ((u.x == kSentinel || u.y == kSentinel || u.z == kSentinel || u.w == kSentinel) && !gave_up) {
                if (++spins > x.spin) {
                    gave_up = true;
                    atomicExch(x.err, 1);
                    break;
                }
                u = ld_volatile_u4(w);
            }
            const float4 v = make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z),
                                         __uint_as_float(u.w));
            s = r == 0 ? v
                       : make_float4(__fadd_rn(s.x, v.x), __fadd_rn(s.y, v.y), __fadd_rn(s.z, v.z), __fadd_rn(s.w, v.w));
            *w = make_uint4(kSentinel, kSentinel, kSentinel, kSentinel);
        }
        reinterpret_cast<float4 *>(buf)[i] = s;
    }
}

}  // namespace

int peer_open(void **out, int rank, int world, int maxn, void *comm, cudaStream_t st)
{
    *out = nullptr;
    if (world < 2 || !comm || maxn % 4) return -1;
    PeerHost *h = new PeerHost();
    h->d.rank = rank;
    h->d.world = world;
    h->d.maxn = maxn;
    h->d.spin = peer_spin_limit();
    const size_t words = (size_t)3 * world * maxn;
    bool ok = cudaMalloc(&h->base, words * 4) == cudaSuccess && cudaMalloc(&h->misc, 4096) == cudaSuccess &&
              cudaMemset(h->misc, 0, 4096) == cudaSuccess;
    if (ok) {
        k_fill_u32<<<256, 256, 0, st>>>(static_cast<unsigned *>(h->base), words, kSentinel);
        ok = cudaStreamSynchronize(st) == cudaSuccess;
    }
    cudaIpcMemHandle_t mine;
    if (ok) ok = cudaIpcGetMemHandle(&mine, h->base) == cudaSuccess;
    // every rank's handle, gathered through NCCL (which also orders every
    // rank's sentinel fill before any exchange)
    std::vector<cudaIpcMemHandle_t> all(world);
    void *dh = nullptr;
    if (ok) ok = cudaMalloc(&dh, sizeof(cudaIpcMemHandle_t) * (world + 1)) == cudaSuccess;
    if (ok) {
        char *d = static_cast<char *>(dh);
        ok = cudaMemcpy(d + sizeof(cudaIpcMemHandle_t) * world, &mine, sizeof mine, cudaMemcpyHostToDevice) ==
                 cudaSuccess &&
             comm_allgather(d + sizeof(cudaIpcMemHandle_t) * world, d, sizeof mine, comm, st) == 0 &&
             cudaStreamSynchronize(st) == cudaSuccess &&
             cudaMemcpy(all.data(), d, sizeof(cudaIpcMemHandle_t) * world, cudaMemcpyDeviceToHost) == cudaSuccess;
    }
    if (dh) cudaFree(dh);
    std::vector<float *> pm(world);
    for (int r = 0; ok && r < world; r++) {
        void *p = h->base;
        if (r != rank) {
            ok = cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
            if (ok) h->opened.push_back(p);
        }
        pm[r] = static_cast<float *>(p);
    }
    if (ok) {
        char *m = static_cast<char *>(h->misc);
        h->d.err = reinterpret_cast<int *>(m);
        float **tm = reinterpret_cast<float **>(m + 64);
        ok = 64 + 8 * world <= 4096 && cudaMemcpy(tm, pm.data(), 8 * world, cudaMemcpyHostToDevice) == cudaSuccess;
        h->d.pmail = tm;
        h->d.mail = static_cast<float *>(h->base);
    }
    if (!ok) {
        fprintf(stderr, "dsv4_b200: peer exchange unavailable (%s); using NCCL\n",
                cudaGetErrorString(cudaGetLastError()));
        peer_close(h);
        return -1;
    }
    *out = h;
    return 0;
}

void peer_close(void *p)
{
    PeerHost *h = static_cast<PeerHost *>(p);
    if (!h) return;
    for (void *q : h->opened) cudaIpcCloseMemHandle(q);
    if (h->base) cudaFree(h->base);
    if (h->misc) cudaFree(h->misc);
    delete h;
}

int peer_allreduce_sum(void *p, float *buf, int n, const unsigned *stepseq, int nx, int call, cudaStream_t st)
{
    PeerHost *h = static_cast<PeerHost *>(p);
    if (!h || n > h->d.maxn || (n & 3) || ((uintptr_t)buf & 15) || !stepseq) return -1;
    const int blocks = 16;
    return launch(k_peer_allreduce, dim3(blocks), dim3(256), 0, st, h->d, buf, n, stepseq, nx, call) == cudaSuccess
               ? 0
               : -1;
}

int xreduce_sum(const Exch &x, float *buf, size_t n, cudaStream_t st)
{
    if (x.peer) return peer_allreduce_sum(x.peer, buf, (int)n, x.stepseq, x.nx, (*x.call)++, st);
    return comm_allreduce_sum(buf, n, x.comm, st);
}

int peer_status(void *p)
{
    PeerHost *h = static_cast<PeerHost *>(p);
    if (!h) return 0;
    int e = 0;
    if (cudaMemcpy(&e, h->d.err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    return e;
}

}  // namespace dsv4b

// One exchange of the peer kernel on ONE GPU with `world` ranks emulated: all
// mailboxes are the same local buffer, rank 0 runs the kernel, and ranks
// 1..world-1 have either stored their vectors beforehand (others_ready) or
// never do (a rank that is gone), which the kernel must survive by giving up
// after spin_limit polls. out[n] receives rank 0's result. Returns the status
// word (0: every rank's values arrived, 1: a wait gave up) or -1.
extern "C" int dsv4b_peer_selftest(int world, int n, unsigned spin_limit, int others_ready, const float *in,
                                   float *out)
{
    using namespace dsv4b;
    if (world < 2 || world > 64 || n <= 0 || (n & 3) || !in || !out || !spin_limit) return -1;
    const size_t words = (size_t)3 * world * n;
    void *mail = nullptr, *misc = nullptr, *buf = nullptr;
    int rc = -1, err = 0;
    PeerDev d = {};
    if (cudaMalloc(&mail, words * 4) != cudaSuccess || cudaMalloc(&misc, 4096) != cudaSuccess ||
        cudaMalloc(&buf, (size_t)n * 4) != cudaSuccess)
        goto done;
    if (cudaMemset(misc, 0, 4096) != cudaSuccess) goto done;
    k_fill_u32<<<64, 256>>>(static_cast<unsigned *>(mail), words, kSentinel);
    if (others_ready) {     // exchange 0 uses buffer 0: ranks 1.. store their slots, -0.0 sent as +0.0
        std::vector<float> v((size_t)(world - 1) * n);
        for (size_t i = 0; i < v.size(); i++) {
            float f = in[(size_t)n + i];
            unsigned u;
            memcpy(&u, &f, 4);
            if (u == kSentinel) f = 0.0f;
            v[i] = f;
        }
        if (cudaMemcpy(static_cast<float *>(mail) + (size_t)n, v.data(), v.size() * 4, cudaMemcpyHostToDevice) !=
            cudaSuccess)
            goto done;
    }
    if (cudaMemcpy(buf, in, (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess) goto done;
    {
        std::vector<float *> pm(world, static_cast<float *>(mail));
        char *m = static_cast<char *>(misc);
        if (64 + 8 * world > 4096 || cudaMemcpy(m + 64, pm.data(), 8 * world, cudaMemcpyHostToDevice) != cudaSuccess)
            goto done;
        d.pmail = reinterpret_cast<float **>(m + 64);
        d.mail = static_cast<float *>(mail);
        d.err = reinterpret_cast<int *>(m);
        d.rank = 0;
        d.world = world;
        d.maxn = n;
        d.spin = spin_limit;
        unsigned *seq = reinterpret_cast<unsigned *>(m + 32);     // step 0 (zeroed above)
        k_peer_allreduce<<<16, 256>>>(d, static_cast<float *>(buf), n, seq, 1, 0);
        if (cudaDeviceSynchronize() != cudaSuccess) goto done;
    }
    if (cudaMemcpy(out, buf, (size_t)n * 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(&err, d.err, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        goto done;
    rc = err;
done:
    if (buf) cudaFree(buf);
    if (misc) cudaFree(misc);
    if (mail) cudaFree(mail);
    return rc;
}
