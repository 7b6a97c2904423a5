// Packed 4-bit weights (sm_100a): the INT8 weights of block mode are Q4_0
// values minus 8, all in [-8, 7], so they pack losslessly two per byte. The
// 4-bit tiled layout keeps the INT8 layout's panels of P columns (fl_layout.cuh)
// with P / 2 bytes per panel row; a 16-byte chunk is one 32-element block in
// the Q4_0 order (gguf_loader.c:147-161): byte j holds q[j] in its low nibble
// and q[j + 16] in its high nibble, q = w + 8 in [0, 15]. The chunks of every
// 128-byte group are XOR-swizzled by (row & 7) like the INT8 layout's. The
// GEMV computes each block's dot over q and subtracts 8 x (sum of the block's
// u8 activations): the same int32 as the INT8 dot.
#include <algorithm>

#include "fl_common.cuh"
#include "fl_kernels.h"
#include "fl_layout.cuh"

namespace fl {

namespace {

// One thread per (row, block): reads the block's 32 int8 weights from the
// INT8 tiled layout and writes its 16 packed bytes; *bad is set when a
// weight lies outside [-8, 7].
__global__ void pack_w4_kernel(const int8_t* __restrict__ w, uint8_t* __restrict__ w4, int N, int K, int P,
                               int* bad) {
    const int nb = K >> 5;
    const size_t total = (size_t)N * nb;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int n = (int)(i / nb), b = (int)(i - (size_t)n * nb);
        const int4 lo = *reinterpret_cast<const int4*>(w + tiled_w_off(N, P, n, 2 * b));
        const int4 hi = *reinterpret_cast<const int4*>(w + tiled_w_off(N, P, n, 2 * b + 1));
        const uint32_t lw[4] = {(uint32_t)lo.x, (uint32_t)lo.y, (uint32_t)lo.z, (uint32_t)lo.w};
        const uint32_t hw[4] = {(uint32_t)hi.x, (uint32_t)hi.y, (uint32_t)hi.z, (uint32_t)hi.w};
        uint32_t out[4];
        bool ok = true;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            uint32_t o = 0;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int a = (int)(int8_t)(lw[k] >> (8 * j));  // element 4k + j
                const int c = (int)(int8_t)(hw[k] >> (8 * j));  // element 16 + 4k + j
                ok = ok && a >= -8 && a <= 7 && c >= -8 && c <= 7;
                o |= (uint32_t)(((a + 8) & 15) | (((c + 8) & 15) << 4)) << (8 * j);
            }
            out[k] = o;
        }
        if (!ok) atomicOr(bad, 1);
        *reinterpret_cast<uint4*>(w4 + tiled_w4_off(N, P, n, b)) = make_uint4(out[0], out[1], out[2], out[3]);
    }
}

}  // namespace

bool w4_supported(int N, int K, int P) { return P > 0 && P % 256 == 0 && K % P == 0 && N % 8 == 0; }

cudaError_t launch_pack_w4(const int8_t* w, uint8_t* w4, int N, int K, int P, int* bad, cudaStream_t s) {
    if (!w4_supported(N, K, P)) return cudaErrorInvalidValue;
    const size_t total = (size_t)N * (K >> 5);
    const int blocks = (int)std::min<size_t>((total + 255) / 256, 148 * 16);
    pack_w4_kernel<<<blocks, 256, 0, s>>>(w, w4, N, K, P, bad);
    return cudaGetLastError();
}

}  // namespace fl
