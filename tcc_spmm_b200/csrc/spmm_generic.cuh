// Generic SpMM kernel: any 2-byte aligned packedX and 4-byte aligned Y/partials. One CTA per
// task and 128-feature slice (grid (tasks, F/128)), four warps of 32 features, operands
// loaded straight from global memory (the layout of the reference kernel,
// src/kernel/spmm_kernel.cuh:172-283). Same arithmetic, write-back and last-arriver merge as
// the persistent kernel; used when the inputs are not 16-byte aligned and as a cross-check.
#pragma once
#include "spmm_common.cuh"

namespace tcc {
namespace {
template <int F>
__global__ void __launch_bounds__(128) spmmGenericKernel(const tcc_sw32_device_view matrix,
                                                         const int8_t* __restrict__ packedX,
                                                         const float* __restrict__ scales,
                                                         float* __restrict__ output, uint32_t rows,
                                                         uint32_t cols, float* __restrict__ partials,
                                                         uint32_t* __restrict__ counters) {
    __shared__ uint32_t lastFlag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t featureBase = blockIdx.y * 128 + warp * 32;
    const tcc_sw32_task task = matrix.tasks[blockIdx.x];
    float acc[4][2][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i)
                acc[r][j][i] = 0.0f;
    for (uint32_t p = task.begin; p < task.end; ++p) {
        const uint32_t m = matrix.rowGroupMasks[p] & 15u;
        uint32_t xf[2][4]; // [part][a0..a3]
        uint32_t mk[2], fv[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) { // slot t (h=0) and t+4 (h=1)
            const uint64_t slot = uint64_t(p) * 8 + t + 4 * h;
            const uint32_t id = matrix.sourceIds[slot];
            const uint64_t meta = matrix.sourceMetadata[slot];
            mk[h] = static_cast<uint32_t>(meta);
            fv[h] = static_cast<uint32_t>(meta >> 32);
            const bool valid = id < cols;
            const float s = valid ? scales[id] : 0.0f;
#pragma unroll
            for (int part = 0; part < 2; ++part) {
                uint32_t pair = 0;
                if (valid)
                    pair = *reinterpret_cast<const unsigned short*>(packedX + uint64_t(id) * F + featureBase +
                                                                    16 * part + 2 * g);
                xf[part][2 * h + 0] = dev::tf32Biased(float(int8_t(pair & 0xFF)) * s);
                xf[part][2 * h + 1] = dev::tf32Biased(float(int8_t(pair >> 8)) * s);
            }
        }
#pragma unroll
        for (int rw = 0; rw < 4; ++rw) {
            if (!(m & (1u << rw)))
                continue;
            const uint32_t bit = 1u << (8 * rw + g);
            uint32_t b[2];
#pragma unroll
            for (int h = 0; h < 2; ++h)
                b[h] = (mk[h] & bit) ? dev::tf32Exact(matrix.values[fv[h] + __popc(mk[h] & (bit - 1))]) : 0u;
#pragma unroll
            for (int part = 0; part < 2; ++part)
                dev::mmaTf32(acc[rw][part], xf[part][0], xf[part][1], xf[part][2], xf[part][3], b[0], b[1]);
        }
    }
    // Fragment (part, i): feature featureBase + 16*part + g + 8*(i>=2), row 8rw + 2t + (i&1).
    if (task.sw == kSkipTask) // a padding entry: no panels, no rows
        return;
    const uint32_t rowBase = task.sw * 32;
    if (task.partial != kNoPartial && (partials == nullptr || counters == nullptr)) {
        if (threadIdx.x == 0) // split tasks need the workspace
            atomicOr(&gDeviceStatus, 2u);
        return;
    }
#pragma unroll
    for (int rw = 0; rw < 4; ++rw)
#pragma unroll
        for (int part = 0; part < 2; ++part)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t row = rowBase + 8 * rw + 2 * t + (i & 1);
                const uint32_t col = featureBase + 16 * part + g + (i >= 2 ? 8 : 0);
                if (row >= rows)
                    continue;
                if (task.partial == kNoPartial) {
                    output[uint64_t(row) * F + col] = acc[rw][part][i];
                } else if (task.mask & (1u << rw)) {
                    const uint64_t block = task.partial + __popc(task.mask & ((1u << rw) - 1));
                    __stcg(partials + (block * 8 + (row & 7)) * F + col, acc[rw][part][i]);
                }
            }
    if (task.partial == kNoPartial)
        return;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const uint32_t ticket =
            dev::ticketIncrement(counters + uint64_t(task.sw) * (F / 128) + blockIdx.y, task.chunks - 1);
        lastFlag = ticket == task.chunks - 1 ? 1u : 0u;
    }
    __syncthreads();
    if (!lastFlag)
        return;
    __threadfence();
    for (uint32_t rw = 0; rw < 4; ++rw) {
        const uint32_t row0 = rowBase + 8 * rw;
        if (row0 >= rows)
            break;
        const tcc_sw32_reduce_range red = matrix.reductions[task.reduceFirst + rw];
        const uint32_t validRows = min(8u, rows - row0);
        for (uint32_t e = threadIdx.x; e < validRows * 128; e += blockDim.x) {
            const uint32_t r = e / 128, col = blockIdx.y * 128 + e % 128;
            float sum = 0.0f;
            for (uint32_t item = red.begin; item < red.end; ++item)
                sum += __ldcg(partials + (uint64_t(matrix.partialIds[item]) * 8 + r) * F + col);
            output[uint64_t(row0 + r) * F + col] = sum;
        }
    }
}
} // namespace
} // namespace tcc
