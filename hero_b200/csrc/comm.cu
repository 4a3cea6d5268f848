// comm.cu -- multi-GPU plumbing: NCCL all-gather of head outputs (C1) and the
// permutation of gathered head blocks back into the reference row layout.
//
// The reference has no distributed backend; this is the B200 build's one
// collective.  NCCL is bound at run time with dlopen("libnccl.so.2") so the
// library shares whichever NCCL the host process already loaded (PyTorch
// ships its own) instead of linking a second copy.
#include <dlfcn.h>
#include <string.h>

#include "common.cuh"

using nmg::set_error;

namespace {

typedef int nccl_result;  // ncclResult_t: 0 = ncclSuccess
typedef void* nccl_comm;  // ncclComm_t
struct nccl_uid {
    char internal[128];
};

struct Nccl {
    void* handle = nullptr;
    nccl_result (*get_unique_id)(nccl_uid*) = nullptr;
    nccl_result (*comm_init_rank)(nccl_comm*, int, nccl_uid, int) = nullptr;
    nccl_result (*comm_destroy)(nccl_comm) = nullptr;
    nccl_result (*all_gather)(const void*, void*, size_t, int, nccl_comm, cudaStream_t) = nullptr;
    const char* (*error_string)(nccl_result) = nullptr;
};

int load_nccl(Nccl** out) {
    static Nccl n;
    static bool tried = false;
    if (!tried) {
        tried = true;
        n.handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (n.handle) {
            n.get_unique_id = (nccl_result(*)(nccl_uid*))dlsym(n.handle, "ncclGetUniqueId");
            n.comm_init_rank = (nccl_result(*)(nccl_comm*, int, nccl_uid, int))dlsym(n.handle, "ncclCommInitRank");
            n.comm_destroy = (nccl_result(*)(nccl_comm))dlsym(n.handle, "ncclCommDestroy");
            n.all_gather = (nccl_result(*)(const void*, void*, size_t, int, nccl_comm, cudaStream_t))dlsym(
                n.handle, "ncclAllGather");
            n.error_string = (const char* (*)(nccl_result))dlsym(n.handle, "ncclGetErrorString");
        }
    }
    if (!n.handle || !n.get_unique_id || !n.comm_init_rank || !n.comm_destroy || !n.all_gather)
        return set_error(NMG_COMM_ERROR, "NCCL (libnccl.so.2) could not be loaded: %s", dlerror() ? dlerror() : "missing symbols");
    *out = &n;
    return NMG_OK;
}

const char* nccl_msg(Nccl* n, nccl_result r) { return n->error_string ? n->error_string(r) : "nccl error"; }

// gathered [world][rows][bytes_per_rank_row] -> out [rows][world][bytes_per_rank_row], 16-byte units.
__global__ void heads_to_rows_kernel(const uint4* __restrict__ in, uint4* __restrict__ out, int world, int64_t rows,
                                     int64_t vecs) {
    const int64_t total = (int64_t)world * rows * vecs;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = t % vecs;
        const int64_t rr = t / vecs;
        const int64_t r = rr % rows;
        const int64_t w = rr / rows;
        out[(r * world + w) * vecs + c] = in[t];
    }
}

__global__ void heads_to_rows_bytes_kernel(const unsigned char* __restrict__ in, unsigned char* __restrict__ out,
                                           int world, int64_t rows, int64_t bytes) {
    const int64_t total = (int64_t)world * rows * bytes;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = t % bytes;
        const int64_t rr = t / bytes;
        const int64_t r = rr % rows;
        const int64_t w = rr / rows;
        out[(r * world + w) * bytes + c] = in[t];
    }
}

}  // namespace

struct nmg_comm {
    Nccl* nccl = nullptr;
    nccl_comm comm = nullptr;
    int rank = 0, world = 1, device = 0;
    unsigned char* bar = nullptr;  // world bytes for the stream-ordered barrier
};

extern "C" int nmg_comm_unique_id(void* id128) {
    if (!id128) return set_error(NMG_INVALID_ARGUMENT, "nmg_comm_unique_id: null buffer");
    Nccl* n = nullptr;
    int st = load_nccl(&n);
    if (st != NMG_OK) return st;
    nccl_uid uid;
    const nccl_result r = n->get_unique_id(&uid);
    if (r != 0) return set_error(NMG_COMM_ERROR, "ncclGetUniqueId: %s", nccl_msg(n, r));
    memcpy(id128, &uid, sizeof(uid));
    return NMG_OK;
}

extern "C" int nmg_comm_init(const void* id128, int rank, int world, int device, nmg_comm** out) {
    if (!id128 || !out) return set_error(NMG_INVALID_ARGUMENT, "nmg_comm_init: null argument");
    if (world <= 0 || rank < 0 || rank >= world) return set_error(NMG_INVALID_ARGUMENT, "nmg_comm_init: bad rank/world");
    *out = nullptr;
    Nccl* n = nullptr;
    int st = load_nccl(&n);
    if (st != NMG_OK) return st;
    NMG_CUDA_TRY(cudaSetDevice(device));
    nccl_uid uid;
    memcpy(&uid, id128, sizeof(uid));
    nmg_comm* c = new nmg_comm();
    c->nccl = n;
    c->rank = rank;
    c->world = world;
    c->device = device;
    if (cudaMalloc(&c->bar, (size_t)world) != cudaSuccess || cudaMemset(c->bar, 0, (size_t)world) != cudaSuccess) {
        delete c;
        return set_error(NMG_CUDA_ERROR, "nmg_comm_init: barrier buffer");
    }
    const nccl_result r = n->comm_init_rank(&c->comm, world, uid, rank);
    if (r != 0) {
        cudaFree(c->bar);
        delete c;
        return set_error(NMG_COMM_ERROR, "ncclCommInitRank: %s", nccl_msg(n, r));
    }
    *out = c;
    return NMG_OK;
}

extern "C" int nmg_comm_destroy(nmg_comm* c) {
    if (!c) return NMG_OK;
    if (c->comm) c->nccl->comm_destroy(c->comm);
    if (c->bar) cudaFree(c->bar);
    delete c;
    return NMG_OK;
}

extern "C" int nmg_comm_barrier(nmg_comm* c, void* stream) {
    if (!c) return set_error(NMG_INVALID_ARGUMENT, "nmg_comm_barrier: null communicator");
    // An in-place one-byte all-gather: it completes on a rank only after every
    // rank has reached it, i.e. after each rank's earlier work on its stream.
    const nccl_result r = c->nccl->all_gather(c->bar + c->rank, c->bar, 1, /*ncclUint8*/ 1, c->comm, (cudaStream_t)stream);
    if (r != 0) return set_error(NMG_COMM_ERROR, "nmg_comm_barrier: %s", nccl_msg(c->nccl, r));
    return NMG_OK;
}

// ---- device buffers shared between the processes of one node (CUDA IPC) ----

extern "C" int nmg_shared_alloc(int64_t bytes, int device, void** ptr, void* handle64) {
    if (!ptr || !handle64 || bytes <= 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_shared_alloc: bad argument");
    *ptr = nullptr;
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    NMG_CUDA_TRY(cudaSetDevice(device));
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, (size_t)bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, (size_t)bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle((cudaIpcMemHandle_t*)handle64, p);
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        return set_error(NMG_CUDA_ERROR, "nmg_shared_alloc: %s", cudaGetErrorString(e));
    }
    *ptr = p;
    return NMG_OK;
}

extern "C" int nmg_shared_free(void* ptr) {
    if (ptr) NMG_CUDA_TRY(cudaFree(ptr));
    return NMG_OK;
}

extern "C" int nmg_ipc_open(const void* handle64, int device, void** ptr) {
    if (!handle64 || !ptr) return set_error(NMG_INVALID_ARGUMENT, "nmg_ipc_open: null argument");
    *ptr = nullptr;
    int prev = 0;
    NMG_CUDA_TRY(cudaGetDevice(&prev));
    NMG_CUDA_TRY(cudaSetDevice(device));
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(NMG_CUDA_ERROR, "nmg_ipc_open: %s", cudaGetErrorString(e));
    return NMG_OK;
}

extern "C" int nmg_ipc_close(void* ptr) {
    if (ptr) NMG_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
    return NMG_OK;
}

extern "C" int nmg_allgather(nmg_comm* c, const void* send, void* recv, int64_t bytes_per_rank, void* stream) {
    if (!c || !send || !recv || bytes_per_rank < 0) return set_error(NMG_INVALID_ARGUMENT, "nmg_allgather: bad argument");
    const nccl_result r = c->nccl->all_gather(send, recv, (size_t)bytes_per_rank, /*ncclUint8*/ 1, c->comm,
                                              (cudaStream_t)stream);
    if (r != 0) return set_error(NMG_COMM_ERROR, "ncclAllGather: %s", nccl_msg(c->nccl, r));
    return NMG_OK;
}

extern "C" int nmg_gather_heads_to_rows(const void* gathered, void* out, int world, int64_t rows,
                                        int64_t row_bytes_per_rank, void* stream) {
    if (!gathered || !out || world <= 0 || rows < 0 || row_bytes_per_rank <= 0)
        return set_error(NMG_INVALID_ARGUMENT, "nmg_gather_heads_to_rows: bad argument");
    if (rows == 0) return NMG_OK;
    const int64_t total = (int64_t)world * rows * row_bytes_per_rank;
    if (row_bytes_per_rank % 16 == 0 && (uintptr_t)gathered % 16 == 0 && (uintptr_t)out % 16 == 0) {
        const int64_t vecs = row_bytes_per_rank / 16;
        const int64_t n = total / 16;
        const int blocks = (int)((n + 255) / 256 < 148 * 8 ? (n + 255) / 256 : 148 * 8);
        heads_to_rows_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((const uint4*)gathered, (uint4*)out, world,
                                                                        rows, vecs);
    } else {
        const int blocks = (int)((total + 255) / 256 < 148 * 8 ? (total + 255) / 256 : 148 * 8);
        heads_to_rows_bytes_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
            (const unsigned char*)gathered, (unsigned char*)out, world, rows, row_bytes_per_rank);
    }
    NMG_CUDA_TRY(cudaGetLastError());
    return NMG_OK;
}
