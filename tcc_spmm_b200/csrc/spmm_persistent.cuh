// Persistent, warp-specialised SpMM kernel (the fast path of launchSpmmInt8).
//
// Grid: one CTA per resident slot (SMs x occupancy). CTA b processes tasks b, b+G, b+2G, ...
// (G = grid size), so at any moment the CTAs of the GPU work on neighbouring 32-row windows
// and the X rows they share stay in L2. Each CTA covers ALL feature slices of its tasks, so
// the SW32 arrays are read once per call at F=256 too.
//
// Warp NC (producer) streams the 4-panel chunks of all the CTA's tasks through three
// asynchronous stages; nothing it does waits on a copy it issued less than several chunks
// earlier:
//   A step  (kALead chunks ahead): cp.async of the chunk's 32 source IDs, 32 metadata words
//           and 4 row-group masks into the A ring.
//   VX step (kVLead chunks ahead): once the A data has landed and the X stage is free: one
//           cp.async.bulk (TMA engine, no multicast) per valid slot gathers the F-byte
//           packed16 source row into the stage, cp.async brings its scale (zero for padding
//           slots), and the chunk's contiguous value range is copied into the V ring.
//   F step  (the current chunk): once the values have landed, the TF32-rounded A values are
//           scattered into m16n8k8 B-fragment order for the chunk's active 8-row groups and
//           the stage is published (mbarrier arrive with release semantics).
// Warps 0..NC-1 (consumers) own FPW features each. Per panel they read their 4 or 8 bytes of
// each of two source rows with one conflict-free shared load each (rows are skewed by 32
// bytes), dequantize in registers (byte permute into the mantissa of 2^23, packed f32x2
// subtract and multiply, +half-ulp TF32 rounding) and issue FPW/16 m16n8k8 TF32 MMAs per
// active 8-row group into register accumulators. At a task boundary they write Y directly
// from the fragments (or the task's partial blocks, followed by the last-arriver merge,
// reference src/kernel/spmm_kernel.cuh:228-282) while the producer already streams the next
// task.
#pragma once
#include "spmm_common.cuh"

namespace tcc {
namespace {

constexpr int kChunk = 4; // panels per chunk: 32 source slots, one per producer lane

template <int F, int FPW> struct Persist {
    static constexpr int kConsumers = F / FPW;
    static constexpr int kThreads = 32 * (kConsumers + 1);
    static constexpr int kParts = FPW / 16;     // m16 tiles per consumer warp
    static constexpr int kLaneBytes = FPW / 8;  // packed bytes of one source per lane (4 or 8)
    static constexpr int kStages = 6;
    static constexpr int kALead = 8, kARing = kALead + 1;
    static constexpr int kVLead = 4, kVRing = kVLead + 1;
    static_assert(kStages >= kVLead + 2, "a VX step must never wait for the chunk being built");
    static constexpr int kVCap = 256;           // floats per V slot; larger chunks read values directly
    static constexpr int kRowStride = F + 32;   // bytes per staged row, 32-byte skew
    static constexpr int kXBytes = 32 * kRowStride;
    static constexpr int kScaleBytes = 32 * 4;
    static constexpr int kFragBytes = kChunk * 4 * 32 * 8;
    static constexpr int kMaskBytes = 16;
    static constexpr int kStageBytes = kXBytes + kScaleBytes + kFragBytes + kMaskBytes;
    static constexpr int kASlotBytes = 128 + 256 + 16 + 16; // ids, metadata, masks, header
    static constexpr int kVSlotBytes = kVCap * 4;
    static constexpr int kAOff = kStages * kStageBytes;
    static constexpr int kVOff = kAOff + kARing * kASlotBytes;
    static constexpr int kVBaseOff = kVOff + kVRing * kVSlotBytes;
    static constexpr int kFlagOff = kVBaseOff + 32;
    static constexpr int kBarOff = kFlagOff + 16;
    static constexpr int kBars = 2 * kStages + kARing + kVRing;
    static constexpr int kBytes = kBarOff + 8 * kBars;
    static_assert(kStageBytes % 16 == 0 && kASlotBytes % 16 == 0 && kBarOff % 8 == 0, "alignment");
    static_assert(kVRing <= 8, "vBase area");
};

// Feature (within the consumer's FPW window) of fragment row g (+8 when hi) of part j: the
// lane's kLaneBytes bytes at g*kLaneBytes hold kLaneBytes/2 packed16 pairs of one tile, one
// pair per part.
template <int FPW> __device__ __forceinline__ int fragFeature(int j, int g, int hi) {
    constexpr int laneBytes = FPW / 8, lanesPerTile = 16 / laneBytes;
    return 16 * (g / lanesPerTile) + (laneBytes / 2) * (g % lanesPerTile) + j + 8 * hi;
}

__device__ __forceinline__ void namedBarrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Walks the chunks of this CTA's tasks (b, b+G, ...), skipping empty tasks. The next task's
// panel range is prefetched when a task is entered.
struct ChunkWalker {
    uint32_t slot, begin, end, next;
    uint32_t nBegin, nEnd;
    bool done;
    __device__ __forceinline__ void load(const tcc_sw32_device_view& m, uint32_t s, uint32_t& b, uint32_t& e) const {
        const uint64_t t = uint64_t(blockIdx.x) + uint64_t(s) * gridDim.x;
        if (t < m.taskCount) {
            b = m.tasks[t].begin;
            e = m.tasks[t].end;
        } else {
            b = e = 0xFFFFFFFFu;
        }
    }
    __device__ __forceinline__ void enter(const tcc_sw32_device_view& m) {
        // Advance from the prefetched task until a non-empty one; prefetch its successor.
        for (;;) {
            if (nBegin == 0xFFFFFFFFu) {
                done = true;
                return;
            }
            begin = nBegin;
            end = nEnd;
            ++slot;
            load(m, slot + 1, nBegin, nEnd);
            if (end > begin)
                break;
        }
        next = begin;
    }
    __device__ __forceinline__ void start(const tcc_sw32_device_view& m) {
        slot = 0xFFFFFFFFu; // enter() increments to 0
        done = false;
        load(m, 0, nBegin, nEnd);
        enter(m);
    }
    __device__ __forceinline__ void advance(const tcc_sw32_device_view& m) {
        next += kChunk;
        if (next >= end)
            enter(m);
    }
};

template <int F, int FPW>
__global__ void __launch_bounds__(Persist<F, FPW>::kThreads)
    spmmPersistentKernel(const tcc_sw32_device_view matrix, const int8_t* __restrict__ packedX,
                         const float* __restrict__ scales, float* __restrict__ output, uint32_t rows,
                         uint32_t cols, float* __restrict__ partials, uint32_t* __restrict__ counters) {
    using L = Persist<F, FPW>;
    extern __shared__ __align__(128) unsigned char smem[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t base = dev::smemAddr(smem);
    const uint32_t barX = base + L::kBarOff;   // stage full   [kStages]
    const uint32_t barE = barX + 8 * L::kStages; // stage empty  [kStages]
    const uint32_t barA = barE + 8 * L::kStages; // A slot landed [kARing]
    const uint32_t barV = barA + 8 * L::kARing;  // V slot landed [kVRing]
    volatile uint32_t* flags = reinterpret_cast<volatile uint32_t*>(smem + L::kFlagOff);
    if (threadIdx.x == 0) {
        for (int s = 0; s < L::kStages; ++s) {
            dev::mbarInit(barX + 8 * s, 64); // 32 cp.async arrivals (scales) + 32 producer arrivals
            dev::mbarInit(barE + 8 * s, L::kConsumers);
        }
        for (int s = 0; s < L::kARing; ++s)
            dev::mbarInit(barA + 8 * s, 32);
        for (int s = 0; s < L::kVRing; ++s)
            dev::mbarInit(barV + 8 * s, 32);
        flags[0] = flags[1] = flags[2] = flags[3] = 0;
        dev::fenceBarrierInit();
    }
    __syncthreads();

    if (warp == L::kConsumers) {
        // ==================================== producer ====================================
        uint32_t* vBase = reinterpret_cast<uint32_t*>(smem + L::kVBaseOff);
        const int pp = lane >> 3, k = lane & 7;
        // Total chunks of this CTA.
        uint32_t total = 0;
        for (uint64_t t = blockIdx.x + uint64_t(lane) * gridDim.x; t < matrix.taskCount; t += 32ull * gridDim.x)
            total += (matrix.tasks[t].end - matrix.tasks[t].begin + kChunk - 1) / kChunk;
        total = __reduce_add_sync(0xFFFFFFFFu, total);
        ChunkWalker walk;
        walk.start(matrix);
        uint32_t seqA = 0, seqV = 0;
        bool ok = true;
        for (uint32_t seqF = 0; seqF < total && ok; ++seqF) {
            // ---- A steps ----
            for (; seqA < total && seqA <= seqF + L::kALead; ++seqA) {
                const uint32_t slot = seqA % L::kARing;
                unsigned char* a = smem + L::kAOff + slot * L::kASlotBytes;
                const uint32_t p0 = walk.next;
                const uint32_t np = min(uint32_t(kChunk), walk.end - p0);
                if (lane == 0) {
                    reinterpret_cast<uint32_t*>(a + 400)[0] = p0;
                    reinterpret_cast<uint32_t*>(a + 400)[1] = np;
                }
                if (uint32_t(pp) < np) {
                    const uint64_t s = uint64_t(p0 + pp) * 8 + k;
                    dev::cpAsync4(dev::smemAddr(a + 4 * lane), matrix.sourceIds + s, 4);
                    dev::cpAsync8(dev::smemAddr(a + 128 + 8 * lane), matrix.sourceMetadata + s);
                }
                if (uint32_t(lane) < np)
                    dev::cpAsync4(dev::smemAddr(a + 384 + 4 * lane), matrix.rowGroupMasks + p0 + lane, 4);
                dev::cpAsyncArriveNoinc(barA + 8 * slot);
                walk.advance(matrix);
            }
            __syncwarp();
            // ---- VX steps: X rows, scales and values of chunks up to seqF + kVLead ----
            for (; seqV < seqA && seqV <= seqF + L::kVLead; ++seqV) {
                const uint32_t aslot = seqV % L::kARing, vslot = seqV % L::kVRing, stage = seqV % L::kStages;
                if (!boundedWait(barA + 8 * aslot, (seqV / L::kARing) & 1) ||
                    (seqV >= L::kStages && !boundedWait(barE + 8 * stage, ((seqV / L::kStages) - 1) & 1))) {
                    ok = false;
                    break;
                }
                const unsigned char* a = smem + L::kAOff + aslot * L::kASlotBytes;
                const uint32_t np = reinterpret_cast<const uint32_t*>(a + 400)[1];
                const bool inRange = uint32_t(pp) < np;
                const uint32_t id = inRange ? *reinterpret_cast<const uint32_t*>(a + 4 * lane) : 0xFFFFFFFFu;
                const uint64_t meta = inRange ? *reinterpret_cast<const uint64_t*>(a + 128 + 8 * lane) : 0ull;
                const bool valid = id < cols;
                unsigned char* st = smem + stage * L::kStageBytes;
                const uint32_t bar = barX + 8 * stage;
                dev::mbarExpectTx(bar, valid ? uint32_t(F) : 0u);
                if (valid)
                    dev::bulkCopyG2S(dev::smemAddr(st + lane * L::kRowStride), packedX + uint64_t(id) * F, F, bar);
                dev::cpAsync4(dev::smemAddr(st + L::kXBytes + 4 * (pp * 8 + 2 * (k & 3) + (k >> 2))),
                              valid ? static_cast<const void*>(scales + id) : static_cast<const void*>(scales),
                              valid ? 4u : 0u);
                dev::cpAsyncArriveNoinc(bar);
                // Values of a chunk are contiguous in slot order.
                const uint32_t mask = static_cast<uint32_t>(meta);
                const uint32_t first = static_cast<uint32_t>(meta >> 32);
                const uint32_t lo = __reduce_min_sync(0xFFFFFFFFu, mask ? first : 0xFFFFFFFFu);
                const uint32_t hi = __reduce_max_sync(0xFFFFFFFFu, mask ? first + __popc(mask) : 0u);
                const uint32_t count = hi > lo ? hi - lo : 0u;
                if (lane == 0)
                    vBase[vslot] = count <= uint32_t(L::kVCap) ? lo : 0xFFFFFFFFu;
                if (count <= uint32_t(L::kVCap)) {
                    unsigned char* v = smem + L::kVOff + vslot * L::kVSlotBytes;
                    for (uint32_t i = lane; i < count; i += 32)
                        dev::cpAsync4(dev::smemAddr(v + 4 * i), matrix.values + lo + i, 4);
                }
                dev::cpAsyncArriveNoinc(barV + 8 * vslot);
            }
            if (!ok)
                break;
            // ---- F step: B fragments and masks of chunk seqF; publish the stage ----
            const uint32_t aslot = seqF % L::kARing, vslot = seqF % L::kVRing, stage = seqF % L::kStages;
            if (!boundedWait(barV + 8 * vslot, (seqF / L::kVRing) & 1)) {
                ok = false;
                break;
            }
            const unsigned char* a = smem + L::kAOff + aslot * L::kASlotBytes;
            const uint32_t np = reinterpret_cast<const uint32_t*>(a + 400)[1];
            unsigned char* st = smem + stage * L::kStageBytes;
            uint32_t* stMask = reinterpret_cast<uint32_t*>(st + L::kXBytes + L::kScaleBytes + L::kFragBytes);
            if (lane < kChunk)
                stMask[lane] = uint32_t(lane) < np ? (*reinterpret_cast<const uint32_t*>(a + 384 + 4 * lane) & 15u) : 0u;
            float* frag = reinterpret_cast<float*>(st + L::kXBytes + L::kScaleBytes);
            {
                uint4* z = reinterpret_cast<uint4*>(frag);
#pragma unroll
                for (int i = 0; i < L::kFragBytes / 16 / 32; ++i)
                    z[i * 32 + lane] = make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
            const uint64_t meta = uint32_t(pp) < np ? *reinterpret_cast<const uint64_t*>(a + 128 + 8 * lane) : 0ull;
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
                frag[((pp * 4 + (bit >> 3)) * 32 + 4 * (bit & 7) + (k & 3)) * 2 + (k >> 2)] =
                    __uint_as_float(dev::tf32Exact(value));
            }
            dev::mbarArrive(barX + 8 * stage);
        }
        if (!ok) {
            flags[1] = 1;
            dev::cpAsyncWaitAll();
        }
    } else {
        // ==================================== consumers ===================================
        const int g = lane >> 2, t = lane & 3;
        const int c = warp;
        uint32_t seq = 0;
        bool ok = true;
        // After a wait runs out (ok == false) the consumers keep walking their tasks without
        // waiting or computing, so every named barrier below is still reached by all of them.
        tcc_sw32_task nextTask{};
        if (blockIdx.x < matrix.taskCount)
            nextTask = matrix.tasks[blockIdx.x];
        for (uint64_t tk = blockIdx.x; tk < matrix.taskCount; tk += gridDim.x) {
            const tcc_sw32_task task = nextTask;
            if (tk + gridDim.x < matrix.taskCount) // prefetch the next task descriptor
                nextTask = matrix.tasks[tk + gridDim.x];
            const uint32_t panelCount = task.end - task.begin;
            const uint32_t nch = (panelCount + kChunk - 1) / kChunk;
            float acc[4][L::kParts][4];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int jj = 0; jj < L::kParts; ++jj)
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        acc[r][jj][i] = 0.0f;
            for (uint32_t ch = 0; ch < nch; ++ch, ++seq) {
                const uint32_t stage = seq % L::kStages;
                if (ok && !boundedWait(barX + 8 * stage, (seq / L::kStages) & 1))
                    ok = false;
                if (!ok)
                    continue;
                const unsigned char* st = smem + stage * L::kStageBytes;
                const float2* sc2 = reinterpret_cast<const float2*>(st + L::kXBytes);
                const float2* frag2 = reinterpret_cast<const float2*>(st + L::kXBytes + L::kScaleBytes);
                const uint32_t* stMask =
                    reinterpret_cast<const uint32_t*>(st + L::kXBytes + L::kScaleBytes + L::kFragBytes);
                const uint32_t inChunk = min(uint32_t(kChunk), panelCount - ch * kChunk);
                for (uint32_t pp = 0; pp < inChunk; ++pp) {
                    const uint32_t m = stMask[pp];
                    const float2 s = sc2[pp * 4 + t];
                    const unsigned long long sa = dev::pack2(s.x, s.x), sb = dev::pack2(s.y, s.y);
                    const unsigned char* rowA = st + (pp * 8 + t) * L::kRowStride + c * FPW + L::kLaneBytes * g;
                    const unsigned char* rowB = rowA + 4 * L::kRowStride;
                    uint32_t da[L::kParts * 2], db[L::kParts * 2]; // dequantized sources t and t+4
                    if constexpr (L::kLaneBytes == 8) {
                        const uint2 wa = *reinterpret_cast<const uint2*>(rowA);
                        const uint2 wb = *reinterpret_cast<const uint2*>(rowB);
                        uint32_t t0[4], t1[4];
                        dev::dequant4(wa.x, sa, t0);
                        dev::dequant4(wa.y, sa, t1);
                        da[0] = t0[0]; da[1] = t0[1]; da[2] = t0[2]; da[3] = t0[3];
                        da[4] = t1[0]; da[5] = t1[1]; da[6] = t1[2]; da[7] = t1[3];
                        dev::dequant4(wb.x, sb, t0);
                        dev::dequant4(wb.y, sb, t1);
                        db[0] = t0[0]; db[1] = t0[1]; db[2] = t0[2]; db[3] = t0[3];
                        db[4] = t1[0]; db[5] = t1[1]; db[6] = t1[2]; db[7] = t1[3];
                    } else {
                        const uint32_t wa = *reinterpret_cast<const uint32_t*>(rowA);
                        const uint32_t wb = *reinterpret_cast<const uint32_t*>(rowB);
                        uint32_t t0[4];
                        dev::dequant4(wa, sa, t0);
                        da[0] = t0[0]; da[1] = t0[1]; da[2] = t0[2]; da[3] = t0[3];
                        dev::dequant4(wb, sb, t0);
                        db[0] = t0[0]; db[1] = t0[1]; db[2] = t0[2]; db[3] = t0[3];
                    }
#pragma unroll
                    for (int rw = 0; rw < 4; ++rw) {
                        if (m & (1u << rw)) {
                            const float2 bf = frag2[(pp * 4 + rw) * 32 + lane];
                            const uint32_t f0 = __float_as_uint(bf.x), f1 = __float_as_uint(bf.y);
#pragma unroll
                            for (int jj = 0; jj < L::kParts; ++jj)
                                dev::mmaTf32(acc[rw][jj], da[2 * jj], da[2 * jj + 1], db[2 * jj], db[2 * jj + 1], f0, f1);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0)
                    dev::mbarArrive(barE + 8 * stage);
            }
            // ---- write-back of this task ----
            const uint32_t rowBase = task.sw * 32;
            const bool split = task.partial != kNoPartial;
            if (split && (partials == nullptr || counters == nullptr)) {
                if (threadIdx.x == 0)
                    atomicOr(&gDeviceStatus, 2u);
                continue;
            }
#pragma unroll
            for (int rw = 0; rw < 4; ++rw) {
                if (split && !(task.mask & (1u << rw)))
                    continue;
                const uint64_t block = split ? task.partial + __popc(task.mask & ((1u << rw) - 1)) : 0;
#pragma unroll
                for (int jj = 0; jj < L::kParts; ++jj)
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t r = 8 * rw + 2 * t + (i & 1);
                        const uint32_t feat = c * FPW + fragFeature<FPW>(jj, g, i >> 1);
                        if (!split) {
                            if (rowBase + r < rows)
                                __stcs(output + uint64_t(rowBase + r) * F + feat, acc[rw][jj][i]);
                        } else {
                            __stcg(partials + (block * 8 + (r & 7)) * F + feat, acc[rw][jj][i]);
                        }
                    }
            }
            if (!split)
                continue;
            // Last-arriver merge among the consumer warps (the producer keeps streaming).
            __threadfence();
            namedBarrier(1, 32 * L::kConsumers);
            if (threadIdx.x == 0 && ok) {
                const uint32_t ticket =
                    dev::ticketIncrement(counters + uint64_t(task.sw) * (F / 128), task.chunks - 1);
                flags[0] = ticket == task.chunks - 1 ? 1u : 0u;
            }
            namedBarrier(1, 32 * L::kConsumers);
            const bool last = ok && flags[0] != 0;
            if (last) {
                __threadfence();
                constexpr uint32_t kVec = F / 4;
                for (uint32_t rw = 0; rw < 4; ++rw) {
                    const uint32_t row0 = rowBase + 8 * rw;
                    if (row0 >= rows)
                        break;
                    const tcc_sw32_reduce_range red = matrix.reductions[task.reduceFirst + rw];
                    const uint32_t validRows = min(8u, rows - row0);
                    for (uint32_t e = threadIdx.x; e < validRows * kVec; e += 32 * L::kConsumers) {
                        const uint32_t r = e / kVec, v = e % kVec;
                        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
                        for (uint32_t item = red.begin; item < red.end; ++item) {
                            const uint64_t blk = matrix.partialIds[item];
                            const float4 p = __ldcg(reinterpret_cast<const float4*>(partials + (blk * 8 + r) * F) + v);
                            sum.x += p.x;
                            sum.y += p.y;
                            sum.z += p.z;
                            sum.w += p.w;
                        }
                        __stcs(reinterpret_cast<float4*>(output + uint64_t(row0 + r) * F) + v, sum);
                    }
                }
            }
            namedBarrier(1, 32 * L::kConsumers); // flags[0] is reused by the next split task
        }
        if (!ok)
            flags[1] = 1;
    }
    __syncthreads();
}

} // namespace
} // namespace tcc
