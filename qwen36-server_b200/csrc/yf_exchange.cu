// Sharded-decode partials exchanged over NVLink peer memory, and their LSE merge.
//
// The sharded long-context decode (kv head x key range per GPU) ends every step with each rank's
// packed partial [O f32 rows*D | lse f32 rows] needed on every rank.  Instead of a collective
// library call, every rank owns an exchange area in its own memory, mapped into the other ranks'
// address spaces once at set-up (CUDA IPC, plain peer mappings); yf_xchg.cuh gives its layout.
// Step s (epoch + 1): this rank's partial is stored into slot `rank` of buffer s & 1 in every
// rank's area with plain stores over NVLink, fenced at system scope, and s is stored into flag
// `rank` of every area (release).  The merge waits (bounded by the exchange's wait limit) until
// every flag of its own area has reached s (acquire), then merges the head groups' parts in place
// into f16 output, as yf_attn_combine does.  Two buffers are enough: a rank writes step s+1 only
// after its merge of step s, which needed every rank's step-s partial, and each rank writes s+1
// only after its own merge of s -- so nobody overwrites a buffer that another rank still reads.
//
// Two ways to run a step: yf_exchange_push then yf_exchange_combine (two kernels after the
// caller's yf_attn_decode_partial; ranks can be emulated on one GPU, every push before every
// combine), or yf_exchange_decode, where the cluster decode kernel itself stores the partial into
// the areas, raises the flags and merges in its last CTA: one launch per step, for ranks on
// separate GPUs only (on one GPU the ranks' kernels would wait on one another).
// Replaces the all-gather + flash_fwd_splitkv_combine_kernel pair
// (docs/plans/2026-09-16-prefil-parity-fa2-and-mmq.md:104-107) across GPUs.
#include <cuda_fp16.h>

#include <cstring>
#include <new>
#include <vector>

#include "yf_device.cuh"
#include "yf_internal.h"
#include "yf_xchg.cuh"

struct yf_exchange {
    int device = -1;
    int rank = 0;
    int world = 1;
    long long slot_floats = 0;
    uint8_t* area = nullptr;        // this rank's area (cudaMalloc)
    size_t area_bytes = 0;
    size_t flags_off = 0;           // byte offset of the meta words (flags, epoch, status)
    size_t sstep_off = 0;           // byte offset of the fused path's slice step counts
    size_t words_off = 0;           // byte offset of the fused path's (value, step) word buffers
    unsigned long long* d_peers = nullptr;  // device array: every rank's area base (own included)
    std::vector<unsigned long long> peers;  // host copy
    std::vector<void*> opened;      // IPC mappings to close
    bool emulated = false;          // a peer area attached in this process on the same device
    float* staging = nullptr;       // the partial of the unfused yf_exchange_decode path
    uint64_t wait_ns = 1000000000ull;
};

namespace yf {
namespace {

constexpr int kXThreads = 256;

struct XParams {
    const unsigned long long* peers;  // area bases
    int rank, world;
    long long slot_floats;
    size_t flags_off;
    uint8_t* local;
};

// One block: this rank's partial into slot `rank` of every area, then its flag in every area.
__global__ void __launch_bounds__(kXThreads) push_kernel(const XParams x, const float4* __restrict__ src) {
    uint32_t* meta = xmeta(x.local, x.flags_off);
    const uint32_t step = meta[x.world] + 1u;  // epoch + 1
    const long long n4 = x.slot_floats / 4;
    for (int k = 0; k < x.world; ++k) {
        float4* dst = reinterpret_cast<float4*>(xslot(x.peers[k], step, x.world, x.slot_floats, x.rank));
        for (long long i = threadIdx.x; i < n4; i += kXThreads) dst[i] = __ldg(src + i);
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        xraise(x.peers, x.world, x.rank, x.flags_off, step);
        meta[x.world] = step;  // the step the combine waits for
    }
}

// Waits (one thread per block) for every rank's flag of the current step, then merges: one
// thread per (head group, row, 4 dims), as xmerge4 describes.
__global__ void __launch_bounds__(kXThreads) exchange_combine_kernel(const XParams x, int n_hg, int n_seq, int rows,
                                                                     int hq, int Hq, int d4n, long long lse_off,
                                                                     uint64_t wait_ns, __half* __restrict__ out) {
    uint32_t* meta = xmeta(x.local, x.flags_off);
    __shared__ int s_ok;
    const uint32_t step = meta[x.world];
    if (threadIdx.x == 0) s_ok = xwait(meta, x.world, step, wait_ns);
    __syncthreads();
    const int e = blockIdx.x * kXThreads + threadIdx.x;
    if (!s_ok || e >= n_hg * rows * d4n) return;
    xmerge4(x.local, step, x.world, x.slot_floats, lse_off, n_hg, n_seq, rows, hq, Hq, d4n, e, out);
}

XParams params_of(const yf_exchange* ex) {
    XParams x;
    x.peers = ex->d_peers;
    x.rank = ex->rank;
    x.world = ex->world;
    x.slot_floats = ex->slot_floats;
    x.flags_off = ex->flags_off;
    x.local = ex->area;
    return x;
}

}  // namespace
}  // namespace yf

using namespace yf;

namespace {

int sync_peers(yf_exchange* ex) {
    const cudaError_t e = cudaMemcpy(ex->d_peers, ex->peers.data(), sizeof(unsigned long long) * ex->world,
                                     cudaMemcpyHostToDevice);
    return e == cudaSuccess ? YF_OK : cuda_fail(e, "peer table upload");
}

}  // namespace

extern "C" {

int yf_exchange_create(int32_t device, int32_t rank, int32_t world, int64_t slot_floats, yf_exchange** out) {
    if (!out) return fail(YF_E_INVALID, "out is null");
    *out = nullptr;
    if (world < 1 || world > 64 || rank < 0 || rank >= world)
        return fail(YF_E_INVALID, "rank %d / world %d (world 1..64)", rank, world);
    if (slot_floats < 4 || slot_floats % 4) return fail(YF_E_INVALID, "slot_floats %lld: a positive multiple of 4",
                                                       (long long)slot_floats);
    yf_exchange* ex = new (std::nothrow) yf_exchange();
    if (!ex) return fail(YF_E_NOMEM, "host allocation failed");
    ex->device = device;
    ex->rank = rank;
    ex->world = world;
    ex->slot_floats = slot_floats;
    ex->flags_off = (size_t)2 * world * slot_floats * sizeof(float);
    ex->sstep_off = ex->flags_off + ((size_t)(world + 2) * sizeof(uint32_t) + 255) / 256 * 256;
    ex->words_off = ex->sstep_off + ((size_t)kXMaxSlices * sizeof(uint32_t) + 255) / 256 * 256;
    ex->area_bytes = ex->words_off + (size_t)2 * world * slot_floats * sizeof(unsigned long long);
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaMalloc(&ex->area, ex->area_bytes);
    if (e == cudaSuccess) e = cudaMemset(ex->area, 0, ex->area_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&ex->d_peers, sizeof(unsigned long long) * world);
    if (e != cudaSuccess) {
        if (ex->area) cudaFree(ex->area);
        delete ex;
        return cuda_fail(e, "exchange area");
    }
    if (e == cudaSuccess) e = cudaMalloc(&ex->staging, (size_t)slot_floats * sizeof(float));
    if (e != cudaSuccess) {
        cudaFree(ex->area);
        cudaFree(ex->d_peers);
        delete ex;
        return cuda_fail(e, "exchange staging");
    }
    ex->peers.assign(world, 0ull);
    ex->peers[rank] = reinterpret_cast<unsigned long long>(ex->area);
    const int rc = sync_peers(ex);
    if (rc) {
        cudaFree(ex->area);
        cudaFree(ex->d_peers);
        delete ex;
        return rc;
    }
    *out = ex;
    return YF_OK;
}

int yf_exchange_destroy(yf_exchange* ex) {
    if (!ex) return YF_OK;
    cudaSetDevice(ex->device);
    for (void* p : ex->opened) cudaIpcCloseMemHandle(p);
    if (ex->staging) cudaFree(ex->staging);
    cudaFree(ex->area);
    cudaFree(ex->d_peers);
    delete ex;
    return YF_OK;
}

int yf_exchange_handle(const yf_exchange* ex, void* out_handle) {
    if (!ex || !out_handle) return fail(YF_E_INVALID, "null argument");
    cudaIpcMemHandle_t h;
    cudaSetDevice(ex->device);
    const cudaError_t e = cudaIpcGetMemHandle(&h, ex->area);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    static_assert(sizeof(h) == YF_EXCHANGE_HANDLE_BYTES, "IPC handle size");
    memcpy(out_handle, &h, sizeof(h));
    return YF_OK;
}

int yf_exchange_open_peer(yf_exchange* ex, int32_t peer, const void* handle) {
    if (!ex || !handle) return fail(YF_E_INVALID, "null argument");
    if (peer < 0 || peer >= ex->world || peer == ex->rank) return fail(YF_E_INVALID, "peer %d", peer);
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    cudaSetDevice(ex->device);
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    ex->opened.push_back(p);
    ex->peers[peer] = reinterpret_cast<unsigned long long>(p);
    return sync_peers(ex);
}

int yf_exchange_attach(yf_exchange* ex, int32_t peer, const yf_exchange* other) {
    if (!ex || !other) return fail(YF_E_INVALID, "null argument");
    if (peer < 0 || peer >= ex->world || peer == ex->rank || other->rank != peer || other->world != ex->world ||
        other->slot_floats != ex->slot_floats)
        return fail(YF_E_INVALID, "peer %d does not match the other exchange", peer);
    if (other->device != ex->device) return fail(YF_E_UNSUPPORTED, "attach needs both areas on one device");
    ex->peers[peer] = reinterpret_cast<unsigned long long>(other->area);
    ex->emulated = true;
    return sync_peers(ex);
}

int yf_exchange_set_wait_limit(yf_exchange* ex, uint32_t wait_limit_us) {
    if (!ex) return fail(YF_E_INVALID, "null argument");
    ex->wait_ns = (uint64_t)(wait_limit_us ? wait_limit_us : 1000000u) * 1000ull;
    return YF_OK;
}

int yf_exchange_push(yf_exchange* ex, const float* d_partial, void* stream) {
    if (!ex || !d_partial) return fail(YF_E_INVALID, "null argument");
    if (!aligned(d_partial, 16)) return fail(YF_E_INVALID, "partial must be 16-byte aligned");
    for (int k = 0; k < ex->world; ++k)
        if (!ex->peers[k]) return fail(YF_E_STATE, "rank %d's area is not mapped", k);
    push_kernel<<<1, kXThreads, 0, static_cast<cudaStream_t>(stream)>>>(params_of(ex),
                                                                      reinterpret_cast<const float4*>(d_partial));
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? YF_OK : cuda_fail(e, "exchange push launch");
}

int yf_exchange_combine(yf_exchange* ex, int32_t n_head_groups, int32_t n_seq, int32_t rows, int32_t hq,
                        int32_t n_q_heads, int32_t head_dim, int64_t lse_offset, void* d_out, void* stream) {
    if (!ex || !d_out) return fail(YF_E_INVALID, "null argument");
    if (n_head_groups < 1 || n_seq < 1 || (long long)n_head_groups * n_seq != ex->world)
        return fail(YF_E_INVALID, "n_head_groups %d x n_seq %d != world %d", n_head_groups, n_seq, ex->world);
    if (rows < 1 || hq < 1 || rows % hq || n_q_heads != hq * n_head_groups)
        return fail(YF_E_INVALID, "rows %d, hq %d, n_q_heads %d", rows, hq, n_q_heads);
    if (head_dim < 4 || head_dim % 4) return fail(YF_E_INVALID, "head_dim %d", head_dim);
    if (lse_offset < (long long)rows * head_dim || lse_offset + rows > ex->slot_floats)
        return fail(YF_E_INVALID, "partial layout exceeds the slot");
    if (!aligned(d_out, 8)) return fail(YF_E_INVALID, "out must be 8-byte aligned");
    const long long n = (long long)n_head_groups * rows * (head_dim / 4);
    const unsigned blocks = (unsigned)((n + kXThreads - 1) / kXThreads);
    exchange_combine_kernel<<<blocks, kXThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        params_of(ex), n_head_groups, n_seq, rows, hq, n_q_heads, head_dim / 4, (long long)lse_offset, ex->wait_ns,
        static_cast<__half*>(d_out));
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? YF_OK : cuda_fail(e, "exchange combine launch");
}

int yf_exchange_decode(yf_exchange* ex, yf_pool* pool, int32_t layer, const void* d_q, int32_t hq,
                       const uint32_t* d_cu_k, const uint32_t* d_block_table, int32_t max_blocks, int32_t batch,
                       int32_t max_seqlen_k, float scale, int32_t n_head_groups, int32_t n_seq, int32_t n_q_heads,
                       void* d_out, void* d_workspace, size_t workspace_bytes, void* stream) {
    if (!ex || !pool) return fail(YF_E_INVALID, "null argument");
    if (n_head_groups < 1 || n_seq < 1 || (long long)n_head_groups * n_seq != ex->world)
        return fail(YF_E_INVALID, "n_head_groups %d x n_seq %d != world %d", n_head_groups, n_seq, ex->world);
    if (hq < 1 || n_q_heads != hq * n_head_groups)
        return fail(YF_E_INVALID, "n_q_heads %d != hq %d x n_head_groups %d", n_q_heads, hq, n_head_groups);
    if (ex->world > 1 && ex->emulated)
        return fail(YF_E_UNSUPPORTED, "ranks attached on one device: run yf_exchange_push and yf_exchange_combine");
    for (int k = 0; k < ex->world; ++k)
        if (!ex->peers[k]) return fail(YF_E_STATE, "rank %d's area is not mapped", k);
    if (pool->desc.device != ex->device) return fail(YF_E_INVALID, "pool and exchange on different devices");
    const int D = pool->desc.head_dim;
    const long long rows = (long long)batch * hq;
    if (batch < 1 || rows * (D + 1) > ex->slot_floats)
        return fail(YF_E_INVALID, "batch %d x hq %d x (head_dim + 1) exceeds the slot of %lld floats", batch, hq,
                    ex->slot_floats);
    XFuse xf;
    xf.peers = ex->d_peers;
    xf.local = ex->area;
    xf.rank = ex->rank;
    xf.world = ex->world;
    xf.slot_floats = ex->slot_floats;
    xf.lse_off = rows * D;
    xf.flags_off = ex->flags_off;
    xf.sstep_off = ex->sstep_off;
    xf.words_off = ex->words_off;
    xf.n_hg = n_head_groups;
    xf.n_seq = n_seq;
    xf.hq = hq;
    xf.n_q_heads = n_q_heads;
    xf.rows = (int)rows;
    xf.out = static_cast<__half*>(d_out);
    xf.wait_ns = ex->wait_ns;
    bool fused = false;
    int rc = decode_exchange(pool, layer, d_q, hq, d_cu_k, d_block_table, max_blocks, batch, max_seqlen_k, scale, xf,
                             d_workspace, workspace_bytes, stream, &fused);
    if (rc || fused) return rc;
    // another schedule took the call: the partial into the staging slot, then push and combine
    rc = yf_attn_decode_partial(pool, layer, d_q, hq, d_cu_k, d_block_table, max_blocks, batch, max_seqlen_k, scale,
                                ex->staging, ex->staging + rows * D, d_workspace, workspace_bytes, stream);
    if (!rc) rc = yf_exchange_push(ex, ex->staging, stream);
    if (!rc)
        rc = yf_exchange_combine(ex, n_head_groups, n_seq, (int32_t)rows, hq, n_q_heads, D, rows * D, d_out, stream);
    return rc;
}

int yf_exchange_status(yf_exchange* ex, uint32_t* out_bits, int clear) {
    if (!ex || !out_bits) return fail(YF_E_INVALID, "null argument");
    cudaSetDevice(ex->device);
    uint32_t* st = reinterpret_cast<uint32_t*>(ex->area + ex->flags_off) + ex->world + 1;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(out_bits, st, sizeof(uint32_t), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear) e = cudaMemset(st, 0, sizeof(uint32_t));
    if (e != cudaSuccess) return cuda_fail(e, "exchange status");
    return YF_OK;
}

}  // extern "C"
