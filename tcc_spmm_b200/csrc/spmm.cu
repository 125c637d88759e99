// Fused Y = A x dequant(X_int8) SpMM over the SW32 panel format, sm_100a.
//
// Replaces the reference kernel spmmInt8Kernel<F> and its launcher (Shixg-cnic/tcc_spmm
// src/kernel/spmm_kernel.cuh:172-283, src/kernel/spmm.cu:1-31) behind the same arrays and
// workspace contract. What is kept from the reference, because the ABI or the numbers depend
// on it: the SW32 panel/task/partial layouts, TF32 operands rounded to nearest with ties away
// from zero, FP32 accumulation on tensor cores, the direct write of unsplit tasks, the
// partial blocks [partialCount][8][F] of split tasks and the last-arriver merge with a
// wrapping acquire-release ticket that returns every counter to zero.
//
// Pipelined kernel (the fast path): one CTA per task and ALL feature slices, so the A-side
// stream (IDs, metadata, masks, values) is read once per task even at F=256.
//   * warp NC (producer) runs three asynchronous stages ahead of the consumers:
//       A-ring : cp.async of the next chunks' source IDs, metadata and row-group masks;
//       V-ring : cp.async of each chunk's contiguous value range;
//       X-stage: one cp.async.bulk (TMA engine) per source slot gathers the F-byte packed16
//                row into shared memory, cp.async brings its scale, and the producer
//                scatters the chunk's TF32-rounded A values into MMA B-fragment order.
//   * warps 0..NC-1 (consumers, 64 features each) read the staged rows with conflict-free
//     8-byte shared loads, dequantize in registers (byte permute + packed f32x2 add/mul +
//     TF32 rounding) and issue m16n8k8 TF32 MMAs into register accumulators for the active
//     8-row groups of each panel only.
//   * Epilogue: accumulators -> shared tile -> coalesced 16-byte stores to Y (unsplit) or
//     to the task's partial blocks, then the last-arriver merge.
// Every wait is bounded (about two seconds of %globaltimer); a wait that runs out records a
// status word and the kernel returns without hanging.
#include "common.hpp"
#include "spmm_device.cuh"

#include <cuda_runtime.h>
#include <mutex>

namespace tcc {

__device__ unsigned int gDeviceStatus = 0;

namespace {

constexpr uint32_t kNoPartial = 0xFFFFFFFFu;
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ bool boundedWait(uint32_t bar, uint32_t parity) {
    if (dev::mbarTryWait(bar, parity))
        return true;
    const uint64_t start = dev::globalTimerNs();
    for (;;) {
        if (dev::mbarTryWait(bar, parity))
            return true;
        if (dev::globalTimerNs() - start > kWaitLimitNs) {
            atomicOr(&gDeviceStatus, 1u);
            return false;
        }
    }
}

// ------------------------------------------------------------------------------------------
// Pipelined kernel configuration and shared-memory layout.
// ------------------------------------------------------------------------------------------
constexpr int kChunk = 4;    // panels per chunk: 32 source slots, one per producer lane
constexpr int kStages = 4;   // X stages in flight
constexpr int kARing = 5;    // A-ring slots (> kALead)
constexpr int kALead = 4;    // A-ring lookahead in chunks
constexpr int kVRing = 3;    // value-ring slots (> kVLead)
constexpr int kVLead = 2;    // value-ring lookahead in chunks
constexpr int kVCap = 256;   // floats per value-ring slot; larger chunks read values directly

template <int F> struct PipeLayout {
    static constexpr int kConsumers = F / 64;
    static constexpr int kThreads = 32 * (kConsumers + 1);
    static constexpr int kRowStride = F + 32;                 // bytes; 32-byte skew per slot
    static constexpr int kXBytes = 32 * kRowStride;           // staged source rows
    static constexpr int kScaleBytes = 32 * 4;                // scales, (s_t, s_t+4) pair order
    static constexpr int kFragBytes = kChunk * 4 * 32 * 8;    // B fragments [panel][rw][lane]
    static constexpr int kMaskBytes = 16;                     // row-group mask per panel
    static constexpr int kStageBytes = kXBytes + kScaleBytes + kFragBytes + kMaskBytes;
    static constexpr int kASlotBytes = 32 * 4 + 32 * 8 + 16;  // ids, metadata, masks
    static constexpr int kVSlotBytes = kVCap * 4;
    static constexpr int kStagesOff = 0;
    static constexpr int kAOff = kStages * kStageBytes;
    static constexpr int kVOff = kAOff + kARing * kASlotBytes;
    static constexpr int kVBaseOff = kVOff + kVRing * kVSlotBytes;  // u32 per V slot
    static constexpr int kFlagOff = kVBaseOff + 16;                 // merge flag, abort flag
    static constexpr int kBarOff = (kFlagOff + 16 + 7) & ~7;
    static constexpr int kBars = 2 * kStages + kARing + kVRing;
    static constexpr int kBytes = kBarOff + kBars * 8;
    static constexpr int kTileStride = F + 4;                       // floats, epilogue tile
    static_assert(32 * kTileStride * 4 <= kStages * kStageBytes, "epilogue tile must fit");
    static_assert(kStageBytes % 16 == 0 && kASlotBytes % 16 == 0, "alignment");
};

// Feature (within a consumer's 64-feature window) of MMA fragment row g (+8 for hi) of
// part j: the consumer's 8-byte load at 8g holds two packed16 pairs of tile g/2, one pair
// per part.
__device__ __forceinline__ int fragFeature(int j, int g, int hi) {
    return 16 * (g >> 1) + 4 * (g & 1) + j + 8 * hi;
}

template <int F>
__global__ void __launch_bounds__(PipeLayout<F>::kThreads, (F == 128 ? 5 : 3))
    spmmPipelinedKernel(const tcc_sw32_device_view matrix, const int8_t* __restrict__ packedX,
                        const float* __restrict__ scales, float* __restrict__ output, uint32_t rows,
                        uint32_t cols, float* __restrict__ partials, uint32_t* __restrict__ counters) {
    using L = PipeLayout<F>;
    extern __shared__ __align__(128) unsigned char smem[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const tcc_sw32_task task = matrix.tasks[blockIdx.x];
    const uint32_t panelCount = task.end - task.begin;
    const uint32_t chunks = (panelCount + kChunk - 1) / kChunk;

    const uint32_t base = dev::smemAddr(smem);
    const uint32_t barX = base + L::kBarOff;                 // full[kStages]
    const uint32_t barE = barX + 8 * kStages;                // empty[kStages]
    const uint32_t barA = barE + 8 * kStages;                // A-ring landed
    const uint32_t barV = barA + 8 * kARing;                 // V-ring landed
    volatile uint32_t* flags = reinterpret_cast<volatile uint32_t*>(smem + L::kFlagOff);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            dev::mbarInit(barX + 8 * s, 64);          // 32 producer arrivals + 32 cp.async arrivals
            dev::mbarInit(barE + 8 * s, L::kConsumers);
        }
        for (int s = 0; s < kARing; ++s)
            dev::mbarInit(barA + 8 * s, 32);
        for (int s = 0; s < kVRing; ++s)
            dev::mbarInit(barV + 8 * s, 32);
        flags[0] = 0;
        flags[1] = 0;
        dev::fenceBarrierInit();
    }
    __syncthreads();

    float acc[4][4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i)
                acc[r][j][i] = 0.0f;

    if (warp == L::kConsumers) {
        // ================================ producer ================================
        uint32_t* vBase = reinterpret_cast<uint32_t*>(smem + L::kVBaseOff);
        const int pp = lane >> 3, k = lane & 7;
        uint32_t nextA = 0, nextV = 0;
        bool ok = true;
        for (uint32_t xc = 0; xc < chunks && ok; ++xc) {
            // A-ring: IDs, metadata and masks of chunks up to xc + kALead.
            for (; nextA < chunks && nextA <= xc + kALead; ++nextA) {
                const uint32_t slot = nextA % kARing;
                unsigned char* a = smem + L::kAOff + slot * L::kASlotBytes;
                const uint32_t p = task.begin + nextA * kChunk + pp;
                if (p < task.end) {
                    const uint64_t s = uint64_t(p) * 8 + k;
                    dev::cpAsync4(dev::smemAddr(a + 4 * lane), matrix.sourceIds + s, 4);
                    dev::cpAsync8(dev::smemAddr(a + 128 + 8 * lane), matrix.sourceMetadata + s);
                }
                if (lane < kChunk && task.begin + nextA * kChunk + lane < task.end)
                    dev::cpAsync4(dev::smemAddr(a + 384 + 4 * lane),
                                  matrix.rowGroupMasks + task.begin + nextA * kChunk + lane, 4);
                dev::cpAsyncArriveNoinc(barA + 8 * slot);
            }
            // V-ring: the value range of chunks up to xc + kVLead.
            for (; nextV < nextA && nextV <= xc + kVLead; ++nextV) {
                const uint32_t aslot = nextV % kARing, vslot = nextV % kVRing;
                if (!boundedWait(barA + 8 * aslot, (nextV / kARing) & 1)) {
                    ok = false;
                    break;
                }
                const unsigned char* a = smem + L::kAOff + aslot * L::kASlotBytes;
                const uint32_t p = task.begin + nextV * kChunk + pp;
                const uint64_t meta =
                    p < task.end ? *reinterpret_cast<const uint64_t*>(a + 128 + 8 * lane) : 0ull;
                const uint32_t mask = static_cast<uint32_t>(meta);
                const uint32_t first = static_cast<uint32_t>(meta >> 32);
                // Values of a chunk are contiguous in slot order: [first of the first
                // non-empty slot, end of the last non-empty slot).
                const uint32_t lo = __reduce_min_sync(0xFFFFFFFFu, mask ? first : 0xFFFFFFFFu);
                const uint32_t hi = __reduce_max_sync(0xFFFFFFFFu, mask ? first + __popc(mask) : 0u);
                const uint32_t count = hi > lo ? hi - lo : 0u;
                if (lane == 0)
                    vBase[vslot] = count <= kVCap ? lo : 0xFFFFFFFFu;
                if (count <= kVCap) {
                    unsigned char* v = smem + L::kVOff + vslot * L::kVSlotBytes;
                    for (uint32_t i = lane; i < count; i += 32)
                        dev::cpAsync4(dev::smemAddr(v + 4 * i), matrix.values + lo + i, 4);
                }
                dev::cpAsyncArriveNoinc(barV + 8 * vslot);
            }
            if (!ok)
                break;
            // X-stage of chunk xc.
            const uint32_t aslot = xc % kARing, vslot = xc % kVRing, stage = xc % kStages;
            if (!boundedWait(barV + 8 * vslot, (xc / kVRing) & 1)) {
                ok = false;
                break;
            }
            if (xc >= kStages && !boundedWait(barE + 8 * stage, ((xc / kStages) - 1) & 1)) {
                ok = false;
                break;
            }
            unsigned char* st = smem + L::kStagesOff + stage * L::kStageBytes;
            const unsigned char* a = smem + L::kAOff + aslot * L::kASlotBytes;
            const uint32_t p = task.begin + xc * kChunk + pp;
            const bool inRange = p < task.end;
            const uint32_t id = inRange ? *reinterpret_cast<const uint32_t*>(a + 4 * lane) : 0xFFFFFFFFu;
            const uint64_t meta = inRange ? *reinterpret_cast<const uint64_t*>(a + 128 + 8 * lane) : 0ull;
            const bool valid = id < cols;
            const uint32_t bar = barX + 8 * stage;
            dev::mbarExpectTx(bar, valid ? uint32_t(F) : 0u);
            if (valid)
                dev::bulkCopyG2S(dev::smemAddr(st + lane * L::kRowStride),
                                 packedX + uint64_t(id) * F, F, bar);
            // Scale pairs: slot k of panel pp goes to [pp][2*(k&3) + (k>>2)].
            dev::cpAsync4(dev::smemAddr(st + L::kXBytes + 4 * (pp * 8 + 2 * (k & 3) + (k >> 2))),
                          valid ? static_cast<const void*>(scales + id) : static_cast<const void*>(scales),
                          valid ? 4u : 0u);
            dev::cpAsyncArriveNoinc(bar);
            // Row-group masks of the chunk's panels.
            uint32_t* stMask = reinterpret_cast<uint32_t*>(st + L::kXBytes + L::kScaleBytes + L::kFragBytes);
            if (lane < kChunk) {
                const bool pin = task.begin + xc * kChunk + lane < task.end;
                stMask[lane] = pin ? (*reinterpret_cast<const uint32_t*>(a + 384 + 4 * lane) & 15u) : 0u;
            }
            // B fragments: clear all [panel][rw] tiles, then scatter this slot's values.
            float* frag = reinterpret_cast<float*>(st + L::kXBytes + L::kScaleBytes);
            {
                uint4* z = reinterpret_cast<uint4*>(frag);
#pragma unroll
                for (int i = 0; i < L::kFragBytes / 16 / 32; ++i)
                    z[i * 32 + lane] = make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
            uint32_t mask = static_cast<uint32_t>(meta);
            const uint32_t first = static_cast<uint32_t>(meta >> 32);
            const uint32_t vb = vBase[vslot];
            const float* vsm = reinterpret_cast<const float*>(smem + L::kVOff + vslot * L::kVSlotBytes);
            uint32_t j = 0;
            while (mask) {
                const int bit = __ffs(mask) - 1;
                mask &= mask - 1;
                const float value = vb != 0xFFFFFFFFu ? vsm[first + j - vb] : __ldg(matrix.values + first + j);
                ++j;
                const int rw = bit >> 3, g = bit & 7;
                frag[((pp * 4 + rw) * 32 + 4 * g + (k & 3)) * 2 + (k >> 2)] = __uint_as_float(dev::tf32Exact(value));
            }
            dev::mbarArrive(bar);
        }
        if (!ok) {
            flags[1] = 1;
            dev::cpAsyncWaitAll();
        }
    } else {
        // ================================ consumers ===============================
        const int g = lane >> 2, t = lane & 3;
        const int c = warp;
        for (uint32_t xc = 0; xc < chunks; ++xc) {
            const uint32_t stage = xc % kStages;
            if (!boundedWait(barX + 8 * stage, (xc / kStages) & 1)) {
                flags[1] = 1;
                break;
            }
            const unsigned char* st = smem + L::kStagesOff + stage * L::kStageBytes;
            const float2* sc2 = reinterpret_cast<const float2*>(st + L::kXBytes);
            const float2* frag2 = reinterpret_cast<const float2*>(st + L::kXBytes + L::kScaleBytes);
            const uint32_t* stMask =
                reinterpret_cast<const uint32_t*>(st + L::kXBytes + L::kScaleBytes + L::kFragBytes);
            const uint32_t inChunk = min(uint32_t(kChunk), panelCount - xc * kChunk);
            for (uint32_t pp = 0; pp < inChunk; ++pp) {
                const uint32_t m = stMask[pp];
                const float2 s = sc2[pp * 4 + t];
                const uint2 xa = *reinterpret_cast<const uint2*>(st + (pp * 8 + t) * L::kRowStride + c * 64 + 8 * g);
                const uint2 xb =
                    *reinterpret_cast<const uint2*>(st + (pp * 8 + t + 4) * L::kRowStride + c * 64 + 8 * g);
                const unsigned long long sa = dev::pack2(s.x, s.x), sb = dev::pack2(s.y, s.y);
                uint32_t a0[4], a1[4], b0[4], b1[4];
                dev::dequant4(xa.x, sa, a0); // parts 0,1 of source t: lo0 hi0 lo1 hi1
                dev::dequant4(xa.y, sa, a1); // parts 2,3 of source t
                dev::dequant4(xb.x, sb, b0); // parts 0,1 of source t+4
                dev::dequant4(xb.y, sb, b1); // parts 2,3 of source t+4
#pragma unroll
                for (int rw = 0; rw < 4; ++rw) {
                    if (m & (1u << rw)) {
                        const float2 bf = frag2[(pp * 4 + rw) * 32 + lane];
                        const uint32_t f0 = __float_as_uint(bf.x), f1 = __float_as_uint(bf.y);
                        dev::mmaTf32(acc[rw][0], a0[0], a0[1], b0[0], b0[1], f0, f1);
                        dev::mmaTf32(acc[rw][1], a0[2], a0[3], b0[2], b0[3], f0, f1);
                        dev::mmaTf32(acc[rw][2], a1[0], a1[1], b1[0], b1[1], f0, f1);
                        dev::mmaTf32(acc[rw][3], a1[2], a1[3], b1[2], b1[3], f0, f1);
                    }
                }
            }
            __syncwarp();
            if (lane == 0)
                dev::mbarArrive(barE + 8 * stage);
        }
    }
    __syncthreads();
    if (flags[1] != 0)
        return; // a wait ran out; the status word says so and Y is not written

    // ================================ epilogue ====================================
    float* tile = reinterpret_cast<float*>(smem + L::kStagesOff);
    if (warp < L::kConsumers) {
        const int g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int rw = 0; rw < 4; ++rw)
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int row = 8 * rw + 2 * t + (i & 1);
                    const int feat = warp * 64 + fragFeature(j, g, i >> 1);
                    tile[row * L::kTileStride + feat] = acc[rw][j][i];
                }
    }
    __syncthreads();
    const uint32_t rowBase = task.sw * 32;
    constexpr int kVec = F / 4;
    if (task.partial == kNoPartial) {
        const uint32_t validRows = min(32u, rows - rowBase);
        for (uint32_t e = threadIdx.x; e < validRows * kVec; e += L::kThreads) {
            const uint32_t r = e / kVec, v = e % kVec;
            const float4 val = *reinterpret_cast<const float4*>(tile + r * L::kTileStride + 4 * v);
            __stcs(reinterpret_cast<float4*>(output + uint64_t(rowBase + r) * F) + v, val);
        }
        return;
    }
    // Split window: write this task's 8-row groups to its private partial blocks.
    if (partials == nullptr || counters == nullptr) { // split tasks need the workspace
        if (threadIdx.x == 0)
            atomicOr(&gDeviceStatus, 2u);
        return;
    }
    for (uint32_t e = threadIdx.x; e < 32 * kVec; e += L::kThreads) {
        const uint32_t r = e / kVec, v = e % kVec, rw = r >> 3;
        if (!(task.mask & (1u << rw)))
            continue;
        const uint64_t block = task.partial + __popc(task.mask & ((1u << rw) - 1));
        const float4 val = *reinterpret_cast<const float4*>(tile + r * L::kTileStride + 4 * v);
        __stcg(reinterpret_cast<float4*>(partials + (block * 8 + (r & 7)) * F) + v, val);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const uint32_t ticket = dev::ticketIncrement(counters + uint64_t(task.sw) * (F / 128), task.chunks - 1);
        flags[0] = ticket == task.chunks - 1 ? 1u : 0u;
    }
    __syncthreads();
    if (flags[0] == 0)
        return;
    __threadfence();
    // Last arriver: sum the window's partial blocks in task order, per 8-row group.
    for (uint32_t rw = 0; rw < 4; ++rw) {
        const uint32_t row0 = rowBase + 8 * rw;
        if (row0 >= rows)
            break;
        const tcc_sw32_reduce_range red = matrix.reductions[task.reduceFirst + rw];
        const uint32_t validRows = min(8u, rows - row0);
        for (uint32_t e = threadIdx.x; e < validRows * kVec; e += L::kThreads) {
            const uint32_t r = e / kVec, v = e % kVec;
            float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
            for (uint32_t item = red.begin; item < red.end; ++item) {
                const uint64_t block = matrix.partialIds[item];
                const float4 p = __ldcg(reinterpret_cast<const float4*>(partials + (block * 8 + r) * F) + v);
                sum.x += p.x;
                sum.y += p.y;
                sum.z += p.z;
                sum.w += p.w;
            }
            __stcs(reinterpret_cast<float4*>(output + uint64_t(row0 + r) * F) + v, sum);
        }
    }
}

// ------------------------------------------------------------------------------------------
// Generic kernel: any 2-byte aligned packedX and 4-byte aligned Y/partials. One CTA per task
// and 128-feature slice (grid (tasks, F/128)), four warps of 32 features, operands loaded
// straight from global memory. Same arithmetic and merge as the pipelined kernel.
// ------------------------------------------------------------------------------------------
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

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

template <int F> void enablePipelined(int device) {
    static std::mutex mutex;
    static bool done[64] = {};
    std::lock_guard<std::mutex> lock(mutex);
    if (device < 0 || device >= 64 || done[device])
        return;
    const cudaError_t s = cudaFuncSetAttribute(spmmPipelinedKernel<F>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               PipeLayout<F>::kBytes);
    if (s != cudaSuccess)
        throw CudaError(cudaGetErrorString(s));
    done[device] = true;
}

template <int F>
void launch(const tcc_sw32_device_view& m, const int8_t* x, const float* scales, float* y, uint32_t rows,
            uint32_t cols, float* partials, uint32_t* counters, cudaStream_t stream, int forceGeneric) {
    const bool fast = !forceGeneric && aligned(x, 16) && aligned(y, 16) && (partials == nullptr || aligned(partials, 16));
    if (fast) {
        int device = 0;
        if (cudaGetDevice(&device) != cudaSuccess)
            throw CudaError("cudaGetDevice failed");
        enablePipelined<F>(device);
        spmmPipelinedKernel<F><<<m.taskCount, PipeLayout<F>::kThreads, PipeLayout<F>::kBytes, stream>>>(
            m, x, scales, y, rows, cols, partials, counters);
    } else {
        spmmGenericKernel<F><<<dim3(m.taskCount, F / 128), 128, 0, stream>>>(m, x, scales, y, rows, cols, partials,
                                                                             counters);
    }
    const cudaError_t status = cudaGetLastError();
    if (status != cudaSuccess)
        throw CudaError(cudaGetErrorString(status));
}

void launchChecked(const tcc_sw32_device_view* matrix, const int8_t* packedX, const float* scales, float* output,
                   uint32_t rows, uint32_t cols, uint32_t features, float* partials, uint32_t* counters,
                   cudaStream_t stream, int forceGeneric) {
    if (matrix == nullptr)
        throw std::invalid_argument("null SW32 device view");
    if (features != 128 && features != 256)
        throw std::invalid_argument("feature dimension must be 128 or 256");
    if (matrix->taskCount == 0) // the reference launches an empty grid (std::runtime_error)
        throw CudaError("invalid configuration argument");
    if (matrix->tasks == nullptr || matrix->sourceIds == nullptr || matrix->sourceMetadata == nullptr ||
        matrix->rowGroupMasks == nullptr || packedX == nullptr || scales == nullptr || output == nullptr)
        throw std::invalid_argument("null device array in launchSpmmInt8");
    if (!aligned(packedX, 2) || !aligned(output, 4))
        throw std::invalid_argument("packedX must be 2-byte and Y 4-byte aligned");
    if (features == 128)
        launch<128>(*matrix, packedX, scales, output, rows, cols, partials, counters, stream, forceGeneric);
    else
        launch<256>(*matrix, packedX, scales, output, rows, cols, partials, counters, stream, forceGeneric);
}

} // namespace
} // namespace tcc

extern "C" {

int tcc_launch_spmm_int8(const tcc_sw32_device_view* matrix, const int8_t* packed_x, const float* scales,
                         float* output, uint32_t rows, uint32_t cols, uint32_t features, float* partials,
                         uint32_t* counters, tcc_stream_t stream) {
    return tcc::guarded([&] {
        tcc::launchChecked(matrix, packed_x, scales, output, rows, cols, features, partials, counters,
                           reinterpret_cast<cudaStream_t>(stream), 0);
    });
}

// Same contract as tcc_launch_spmm_int8 but always runs the generic kernel (kept for tests
// and for comparing the two code paths; not part of the public header).
int tcc_launch_spmm_int8_generic(const tcc_sw32_device_view* matrix, const int8_t* packed_x, const float* scales,
                                 float* output, uint32_t rows, uint32_t cols, uint32_t features, float* partials,
                                 uint32_t* counters, tcc_stream_t stream) {
    return tcc::guarded([&] {
        tcc::launchChecked(matrix, packed_x, scales, output, rows, cols, features, partials, counters,
                           reinterpret_cast<cudaStream_t>(stream), 1);
    });
}

int tcc_device_status(uint32_t* status, int reset) {
    return tcc::guarded([&] {
        if (status == nullptr)
            throw std::invalid_argument("null status");
        cudaError_t s = cudaDeviceSynchronize();
        if (s == cudaSuccess)
            s = cudaMemcpyFromSymbol(status, tcc::gDeviceStatus, sizeof(uint32_t));
        if (s == cudaSuccess && reset) {
            const uint32_t zero = 0;
            s = cudaMemcpyToSymbol(tcc::gDeviceStatus, &zero, sizeof(uint32_t));
        }
        if (s != cudaSuccess)
            throw tcc::CudaError(cudaGetErrorString(s));
    });
}

} // extern "C"
