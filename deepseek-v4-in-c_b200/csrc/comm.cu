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
#include <string.h>

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
