// LSE merge of sharded decode partials (yf_attn_combine): the cross-GPU counterpart of the
// reference's flash_fwd_splitkv_combine_kernel
// (docs/plans/2026-09-16-prefil-parity-fa2-and-mmq.md:104-107).  The partials come from
// yf_attn_decode_partial on each shard and reach this GPU by an all-gather.
#include <cuda_fp16.h>

#include "yf_device.cuh"
#include "yf_internal.h"

namespace yf {
namespace {

constexpr int kCombineThreads = 256;

// One thread per (row, 4 dims): out = sum_k w_k o_k / sum_k w_k with w_k = e^(lse_k - max lse).
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const float* __restrict__ o, long long os,
                                                                  const float* __restrict__ lse, long long ls,
                                                                  int n_parts, int rows, int d4n,
                                                                  __half* __restrict__ out) {
    const int e = blockIdx.x * kCombineThreads + threadIdx.x;
    if (e >= rows * d4n) return;
    const int r = e / d4n, c = e % d4n;
    float M = -INFINITY;
    for (int k = 0; k < n_parts; ++k) M = fmaxf(M, __ldg(lse + k * ls + r));
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (M != -INFINITY) {
        for (int k = 0; k < n_parts; ++k) {
            const float lv = __ldg(lse + k * ls + r);
            if (lv == -INFINITY) continue;
            const float w = fast_exp2((lv - M) * 1.4426950408889634f);
            L += w;
            const float4 v = __ldg(reinterpret_cast<const float4*>(o + k * os) + (size_t)r * d4n + c);
            acc.x = fmaf(w, v.x, acc.x);
            acc.y = fmaf(w, v.y, acc.y);
            acc.z = fmaf(w, v.z, acc.z);
            acc.w = fmaf(w, v.w, acc.w);
        }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    uint2 pk;
    pk.x = pack_h2(acc.x * inv, acc.y * inv);
    pk.y = pack_h2(acc.z * inv, acc.w * inv);
    reinterpret_cast<uint2*>(out)[e] = pk;
}

}  // namespace
}  // namespace yf

extern "C" int yf_attn_combine(const float* o_parts, int64_t o_part_stride, const float* lse_parts,
                               int64_t lse_part_stride, int32_t n_parts, int32_t rows, int32_t head_dim, void* out,
                               void* stream) {
    using namespace yf;
    if (rows < 0 || n_parts < 1) return fail(YF_E_INVALID, "rows %d < 0 or n_parts %d < 1", rows, n_parts);
    if (head_dim < 4 || head_dim % 4) return fail(YF_E_INVALID, "head_dim %d is not a positive multiple of 4", head_dim);
    if (rows == 0) return YF_OK;
    if (!o_parts || !lse_parts || !out) return fail(YF_E_INVALID, "null device pointer");
    if (o_part_stride < 0 || lse_part_stride < 0 || o_part_stride % 4)
        return fail(YF_E_INVALID, "part strides must be >= 0 and the O stride a multiple of 4 floats");
    if (!aligned(o_parts, 16) || !aligned(out, 8) || !aligned(lse_parts, 4))
        return fail(YF_E_INVALID, "o_parts 16-byte, out 8-byte and lse 4-byte alignment required");
    const long long n = (long long)rows * (head_dim / 4);
    if (n > 0x7fffffffLL) return fail(YF_E_UNSUPPORTED, "combine of %d rows x %d too large", rows, head_dim);
    const unsigned blocks = (unsigned)((n + kCombineThreads - 1) / kCombineThreads);
    combine_kernel<<<blocks, kCombineThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        o_parts, (long long)o_part_stride, lse_parts, (long long)lse_part_stride, n_parts, rows, head_dim / 4,
        static_cast<__half*>(out));
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? YF_OK : cuda_fail(e, "combine launch");
}
