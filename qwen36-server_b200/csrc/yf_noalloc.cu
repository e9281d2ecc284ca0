// Decode attention for callers that cannot allocate device memory.
//
// yf_attn_decode needs a split-KV workspace from the caller.  Some callers
// have no way to provide one: their device memory is planned once at start-up
// and handed out by an allocator they do not control from the FFI layer (the
// engine's VRAM planner divides the card between weights and the KV pool
// before serving starts), and calling cudaMalloc themselves would go around
// that budget and can fail, or synchronise the device, in the middle of a
// request.  yf_attn_decode_noalloc runs the same kernels with the partials in
// a fixed-size array that is part of this library's device image, so the
// call allocates nothing.
//
// The array lives in every GPU context that loads the library, until the
// process exits.  All calls share it: two calls whose kernels overlap on the
// GPU (different streams, or different host threads on one device) race on
// it and must be serialised by the caller.  Nothing in it needs clearing:
// every partial a call reads was written earlier in the same call.
#include <mutex>

#include "yf_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)16 << 20;  // 16 MiB per device

static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_decode_scratch on `device`, looked up once per device
// with that device current (the host-side name is only a stand-in).
int scratch_address(int device, void** out) {
    if (device < 0 || device >= kMaxDevices) return yf::fail(YF_E_UNSUPPORTED, "device %d out of range", device);
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_addr[device]) {
        int prev = -1;
        cudaError_t e = cudaGetDevice(&prev);
        if (e != cudaSuccess) return yf::cuda_fail(e, "cudaGetDevice");
        if (prev != device) {
            e = cudaSetDevice(device);
            if (e != cudaSuccess) return yf::cuda_fail(e, "cudaSetDevice");
        }
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (prev != device) cudaSetDevice(prev);
        if (e != cudaSuccess) return yf::cuda_fail(e, "cudaGetSymbolAddress(decode scratch)");
        g_scratch_addr[device] = p;
    }
    *out = g_scratch_addr[device];
    return YF_OK;
}

}  // namespace

extern "C" int yf_attn_decode_noalloc(yf_pool* pool, int32_t layer, const void* d_q, int32_t n_q_heads,
                                      const uint32_t* d_cu_seqlens_k, const uint32_t* d_block_table,
                                      int32_t max_blocks, int32_t batch, int32_t max_seqlen_k, float scale,
                                      void* d_out, void* stream) {
    if (!pool) return yf::fail(YF_E_INVALID, "pool is null");
    if (!pool->base) return yf::fail(YF_E_INVALID, "host-only pool has no device memory");
    const size_t need = yf_attn_workspace_size(pool, n_q_heads, batch, 1, max_seqlen_k);
    if (need > kNoAllocScratchBytes)
        return yf::fail(YF_E_WORKSPACE,
                        "this decode needs %zu bytes of split-KV scratch; the built-in scratch holds %zu "
                        "(use yf_attn_decode with a caller workspace)",
                        need, kNoAllocScratchBytes);
    void* scratch = nullptr;
    const int rc = scratch_address(pool->desc.device, &scratch);
    if (rc) return rc;
    return yf_attn_decode(pool, layer, d_q, n_q_heads, d_cu_seqlens_k, d_block_table, max_blocks, batch,
                          max_seqlen_k, scale, d_out, scratch, kNoAllocScratchBytes, stream);
}
