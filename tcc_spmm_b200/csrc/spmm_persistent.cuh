// Persistent, warp-specialised SpMM kernel (the fast path of launchSpmmInt8).
//
// Grid: one CTA per resident slot (SMs x occupancy). CTA b processes tasks b, b+G, b+2G, ...
// (G = grid size), so at any moment the CTAs of the GPU work on neighbouring 32-row windows
// and the feature rows they share stay in L2. Each CTA covers ALL feature slices of its tasks,
// so the SW32 arrays are read once per call at F=256 too.
//
// The chunks (4 panels = 32 source slots) of all the CTA's tasks form one stream that three
// roles work through at different distances:
//   producer warp, A step  (kALead chunks ahead): cp.async of the chunk's 32 source IDs,
//       32 metadata words and 4 row-group masks into the A ring (L2 evict-first: the format is
//       read once).
//   producer warp, V step  (kVLead chunks ahead): cp.async of the chunk's contiguous value
//       range and of its 32 scales into the V ring.
//   consumer warps, X step (kPrefetch chunks ahead): every consumer warp gathers its own
//       FPW-byte slice of the chunk's 32 packed16 source rows with 16-byte cp.async (L2
//       evict-last plus a 128-byte L2 prefetch: the rows are reused by neighbouring windows),
//       tracked by its own cp.async groups.
//   producer warp, F step  (the chunk to be consumed next): the TF32-rounded A values are
//       scattered into m16n8k8 B-fragment order for the chunk's active 8-row groups, the
//       scales into (s_t, s_t+4) pair order, and the stage is published (mbarrier arrive with
//       release semantics).
// Consumers then read their bytes of two source rows per panel with one conflict-free shared
// load each, dequantize in registers (byte permute into the mantissa of 2^23, packed f32x2
// subtract and multiply, +half-ulp TF32 rounding) and issue FPW/16 m16n8k8 TF32 MMAs per
// active 8-row group into register accumulators. At a task boundary they write Y directly
// from the fragments (or the task's partial blocks, followed by the last-arriver merge,
// reference src/kernel/spmm_kernel.cuh:228-282) while the producer streams the next task.
// Every mbarrier wait is bounded (about two seconds).
#pragma once
#include "spmm_common.cuh"

namespace tcc {
namespace {

constexpr int kChunk = 4; // panels per chunk: 32 source slots, one per producer lane

template <int F, int FPW, int P> struct Persist {
    static constexpr int kConsumers = F / FPW;
    static constexpr int kProducers = P;
    static constexpr int kThreads = 32 * (kConsumers + kProducers);
    static constexpr int kParts = FPW / 16;    // m16 tiles per consumer warp
    static constexpr int kLaneBytes = FPW / 8; // packed bytes of one source per lane (4 or 8)
    // Consumer X ring (per consumer warp): kPrefetch chunks in flight plus the one computed.
    // Ring sizes are powers of two (slot = sequence & (size - 1)).
    static constexpr int kXDepth = 4;
    static constexpr int kPrefetch = kXDepth - 1;
    static constexpr int kXRowStride = FPW == 32 ? 32 : 96; // bytes; conflict-free row loads
    static constexpr int kXSlotBytes = 32 * kXRowStride;
    // Producer stages (fragments, scales, masks of one chunk). Scales are stored per panel and
    // fragment column t as (s_t, s_t, s_t+4, s_t+4), ready for the packed f32x2 multiply.
    static constexpr int kStages = 4;
    static constexpr int kScaleBytes = kChunk * 4 * 16;
    static constexpr int kFragBytes = kChunk * 4 * 32 * 8;
    static constexpr int kMaskBytes = 16;
    static constexpr int kStageBytes = kScaleBytes + kFragBytes + kMaskBytes;
    static constexpr int kALead = 6, kARing = 8;
    static constexpr int kVLead = 3, kVRing = 4;
    static_assert(kARing >= kALead + 2 && kVRing >= kVLead + 1, "ring sizes");
    static_assert(kARing % P == 0 && kVRing % P == 0 && kStages % P == 0, "every ring slot has one producer");
    static_assert((kARing & (kARing - 1)) == 0 && (kVRing & (kVRing - 1)) == 0 && (kStages & (kStages - 1)) == 0 &&
                      (kXDepth & (kXDepth - 1)) == 0,
                  "power-of-two rings");
    static constexpr int kVCap = 256;          // values per V slot; larger chunks read them directly
    static constexpr int kASlotBytes = 128 + 256 + 16 + 16; // ids, metadata, masks, header
    static constexpr int kVSlotBytes = kVCap * 4 + 128;     // values, scales
    static constexpr int kXOff = 0;
    static constexpr int kStageOff = kXOff + kConsumers * kXDepth * kXSlotBytes;
    static constexpr int kAOff = kStageOff + kStages * kStageBytes;
    static constexpr int kVOff = kAOff + kARing * kASlotBytes;
    static constexpr int kVBaseOff = kVOff + kVRing * kVSlotBytes;
    static constexpr int kFlagOff = kVBaseOff + 32;
    static constexpr int kBarOff = kFlagOff + 16;
    // xFull[kStages], xEmpty[kStages], aFull[kARing], aUsed[kARing], vFull[kVRing]
    static constexpr int kBars = 2 * kStages + 2 * kARing + kVRing;
    static constexpr int kBytes = kBarOff + 8 * kBars;
    static_assert(kPrefetch <= kALead, "consumers prefetch only chunks whose IDs are requested");
    static_assert(kStageBytes % 16 == 0 && kASlotBytes % 16 == 0 && kVSlotBytes % 16 == 0, "alignment");
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
template <int CH> struct ChunkWalkerT {
    uint32_t slot, begin, end, next;
    uint32_t nBegin, nEnd;
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
        for (;;) {
            if (nBegin == 0xFFFFFFFFu)
                return;
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
        begin = end = next = 0;
        load(m, 0, nBegin, nEnd);
        enter(m);
    }
    __device__ __forceinline__ void advance(const tcc_sw32_device_view& m) {
        next += CH;
        if (next >= end)
            enter(m);
    }
};

// Chunks of CH panels of this CTA (computed by every warp).
template <int CH> __device__ __forceinline__ uint32_t ctaChunkCountT(const tcc_sw32_device_view& m, int lane) {
    uint32_t total = 0;
    for (uint64_t t = blockIdx.x + uint64_t(lane) * gridDim.x; t < m.taskCount; t += 32ull * gridDim.x)
        total += (m.tasks[t].end - m.tasks[t].begin + CH - 1) / CH;
    return __reduce_add_sync(0xFFFFFFFFu, total);
}
using ChunkWalker = ChunkWalkerT<kChunk>;
__device__ __forceinline__ uint32_t ctaChunkCount(const tcc_sw32_device_view& m, int lane) {
    return ctaChunkCountT<kChunk>(m, lane);
}

// Consumer X step: gather warp c's FPW-byte slice of the 32 source rows of chunk s into its X
// ring (16-byte cp.async pieces, padding slots zero-filled) as one cp.async group, then tell the
// producer that the chunk's A slot has been read. Returns false when the A wait ran out.
template <int F, int FPW, int P>
__device__ __forceinline__ bool gatherRows(unsigned char* smem, unsigned char* xring, uint32_t barA, uint32_t barU,
                                           const int8_t* __restrict__ packedX, uint32_t cols, uint32_t total,
                                           uint32_t s, int lane, int c, uint64_t policy, bool ok) {
    using L = Persist<F, FPW, P>;
    if (ok && s < total) {
        const uint32_t aslot = s % L::kARing;
        if (!boundedWait(barA + 8 * aslot, (s / L::kARing) & 1)) {
            ok = false;
        } else {
            const unsigned char* a = smem + L::kAOff + aslot * L::kASlotBytes;
            const uint32_t np = reinterpret_cast<const uint32_t*>(a + 400)[1];
            unsigned char* dst = xring + (s % L::kXDepth) * L::kXSlotBytes;
            constexpr int kPieces = FPW / 16, kRowsPerPass = 32 / kPieces;
#pragma unroll
            for (int pass = 0; pass < kPieces; ++pass) {
                const int row = pass * kRowsPerPass + lane / kPieces, piece = lane % kPieces;
                const uint32_t id = uint32_t(row >> 3) < np ? reinterpret_cast<const uint32_t*>(a)[row] : 0xFFFFFFFFu;
                const bool valid = id < cols;
                dev::cpAsync16Hint(dev::smemAddr(dst + row * L::kXRowStride + 16 * piece),
                                   valid ? static_cast<const void*>(packedX + uint64_t(id) * F + c * FPW + 16 * piece)
                                         : static_cast<const void*>(packedX),
                                   valid ? 16u : 0u, policy);
            }
            __syncwarp();
            if (lane == 0)
                dev::mbarArrive(barU + 8 * aslot);
        }
    }
    dev::cpAsyncCommit();
    return ok;
}

template <int F, int FPW, int P>
__global__ void __launch_bounds__(Persist<F, FPW, P>::kThreads)
    spmmPersistentKernel(const tcc_sw32_device_view matrix, const int8_t* __restrict__ packedX,
                         const float* __restrict__ scales, float* __restrict__ output, uint32_t rows,
                         uint32_t cols, float* __restrict__ partials, uint32_t* __restrict__ counters) {
    using L = Persist<F, FPW, P>;
    extern __shared__ __align__(128) unsigned char smem[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t base = dev::smemAddr(smem);
    const uint32_t barX = base + L::kBarOff;          // stage full    [kStages]
    const uint32_t barE = barX + 8 * L::kStages;      // stage empty   [kStages]
    const uint32_t barA = barE + 8 * L::kStages;      // A slot landed [kARing]
    const uint32_t barU = barA + 8 * L::kARing;       // A slot read by all consumers [kARing]
    const uint32_t barV = barU + 8 * L::kARing;       // V slot landed [kVRing]
    volatile uint32_t* flags = reinterpret_cast<volatile uint32_t*>(smem + L::kFlagOff);
    if (threadIdx.x == 0) {
        for (int s = 0; s < L::kStages; ++s) {
            dev::mbarInit(barX + 8 * s, 32);
            dev::mbarInit(barE + 8 * s, L::kConsumers);
        }
        for (int s = 0; s < L::kARing; ++s) {
            dev::mbarInit(barA + 8 * s, 32);
            dev::mbarInit(barU + 8 * s, L::kConsumers);
        }
        for (int s = 0; s < L::kVRing; ++s)
            dev::mbarInit(barV + 8 * s, 32);
        flags[0] = flags[1] = flags[2] = flags[3] = 0;
        dev::fenceBarrierInit();
    }
    __syncthreads();
    const uint32_t total = ctaChunkCount(matrix, lane);

    if (warp >= L::kConsumers) {
        // ==================================== producers ===================================
        // Producer pw owns the chunks pw, pw+P, pw+2P, ... and every ring slot they map to.
        const uint64_t polStream = dev::policyEvictFirst();
        const uint64_t polKeep = dev::policyEvictLast();
        uint32_t* vBase = reinterpret_cast<uint32_t*>(smem + L::kVBaseOff);
        const int pp = lane >> 3, k = lane & 7;
        const uint32_t pw = warp - L::kConsumers;
        ChunkWalker walk;
        walk.start(matrix);
        for (uint32_t i = 0; i < pw; ++i)
            walk.advance(matrix);
        uint32_t seqA = pw, seqV = pw;
        bool ok = true;
        for (uint32_t seqF = pw; seqF < total && ok; seqF += P) {
            // ---- A steps: IDs, metadata, masks of chunks up to seqF + kALead ----
            for (; seqA < total && seqA <= seqF + L::kALead; seqA += P) {
                const uint32_t slot = seqA % L::kARing;
                if (seqA >= uint32_t(L::kARing) &&
                    !boundedWait(barU + 8 * slot, ((seqA / L::kARing) - 1) & 1)) {
                    ok = false;
                    break;
                }
                unsigned char* a = smem + L::kAOff + slot * L::kASlotBytes;
                const uint32_t p0 = walk.next;
                const uint32_t np = min(uint32_t(kChunk), walk.end - p0);
                if (lane == 0) {
                    reinterpret_cast<uint32_t*>(a + 400)[0] = p0;
                    reinterpret_cast<uint32_t*>(a + 400)[1] = np;
                }
                if (uint32_t(pp) < np) {
                    const uint64_t s = uint64_t(p0 + pp) * 8 + k;
                    dev::cpAsync4Hint(dev::smemAddr(a + 4 * lane), matrix.sourceIds + s, 4, polStream);
                    dev::cpAsync8Hint(dev::smemAddr(a + 128 + 8 * lane), matrix.sourceMetadata + s, polStream);
                }
                if (uint32_t(lane) < np)
                    dev::cpAsync4Hint(dev::smemAddr(a + 384 + 4 * lane), matrix.rowGroupMasks + p0 + lane, 4,
                                      polStream);
                dev::cpAsyncArriveNoinc(barA + 8 * slot);
#pragma unroll
                for (int i = 0; i < P; ++i)
                    walk.advance(matrix);
            }
            if (!ok)
                break;
            __syncwarp();
            // ---- V steps: value ranges and scales of chunks up to seqF + kVLead ----
            for (; seqV < seqA && seqV <= seqF + L::kVLead; seqV += P) {
                const uint32_t aslot = seqV % L::kARing, vslot = seqV % L::kVRing;
                if (!boundedWait(barA + 8 * aslot, (seqV / L::kARing) & 1)) {
                    ok = false;
                    break;
                }
                const unsigned char* a = smem + L::kAOff + aslot * L::kASlotBytes;
                unsigned char* v = smem + L::kVOff + vslot * L::kVSlotBytes;
                const uint32_t np = reinterpret_cast<const uint32_t*>(a + 400)[1];
                const bool inRange = uint32_t(pp) < np;
                const uint32_t id = inRange ? *reinterpret_cast<const uint32_t*>(a + 4 * lane) : 0xFFFFFFFFu;
                const uint64_t meta = inRange ? *reinterpret_cast<const uint64_t*>(a + 128 + 8 * lane) : 0ull;
                const bool valid = id < cols;
                dev::cpAsync4Hint(dev::smemAddr(v + 4 * L::kVCap + 4 * lane),
                                  valid ? static_cast<const void*>(scales + id) : static_cast<const void*>(scales),
                                  valid ? 4u : 0u, polKeep);
                // Values of a chunk are contiguous in slot order.
                const uint32_t mask = static_cast<uint32_t>(meta);
                const uint32_t first = static_cast<uint32_t>(meta >> 32);
                const uint32_t lo = __reduce_min_sync(0xFFFFFFFFu, mask ? first : 0xFFFFFFFFu);
                const uint32_t hi = __reduce_max_sync(0xFFFFFFFFu, mask ? first + __popc(mask) : 0u);
                const uint32_t count = hi > lo ? hi - lo : 0u;
                if (lane == 0)
                    vBase[vslot] = count <= uint32_t(L::kVCap) ? lo : 0xFFFFFFFFu;
                if (count <= uint32_t(L::kVCap))
                    for (uint32_t i = lane; i < count; i += 32)
                        dev::cpAsync4Hint(dev::smemAddr(v + 4 * i), matrix.values + lo + i, 4, polStream);
                dev::cpAsyncArriveNoinc(barV + 8 * vslot);
            }
            if (!ok)
                break;
            // ---- F step: fragments, scales and masks of chunk seqF; publish the stage ----
            const uint32_t aslot = seqF % L::kARing, vslot = seqF % L::kVRing, stage = seqF % L::kStages;
            if (!boundedWait(barV + 8 * vslot, (seqF / L::kVRing) & 1) ||
                (seqF >= uint32_t(L::kStages) && !boundedWait(barE + 8 * stage, ((seqF / L::kStages) - 1) & 1))) {
                ok = false;
                break;
            }
            const unsigned char* a = smem + L::kAOff + aslot * L::kASlotBytes;
            const unsigned char* v = smem + L::kVOff + vslot * L::kVSlotBytes;
            const uint32_t np = reinterpret_cast<const uint32_t*>(a + 400)[1];
            unsigned char* st = smem + L::kStageOff + stage * L::kStageBytes;
            float* stScale = reinterpret_cast<float*>(st);
            float* frag = reinterpret_cast<float*>(st + L::kScaleBytes);
            uint32_t* stMask = reinterpret_cast<uint32_t*>(st + L::kScaleBytes + L::kFragBytes);
            // scale of slot k of panel pp -> both halves of pair (k>>2) of entry [pp][k&3]:
            // consumer lane t reads (s_t, s_t, s_t+4, s_t+4) with one 16-byte load
            {
                const float sk = reinterpret_cast<const float*>(v + 4 * L::kVCap)[lane];
                *reinterpret_cast<float2*>(stScale + (pp * 4 + (k & 3)) * 4 + 2 * (k >> 2)) = make_float2(sk, sk);
            }
            if (lane < kChunk)
                stMask[lane] =
                    uint32_t(lane) < np ? (*reinterpret_cast<const uint32_t*>(a + 384 + 4 * lane) & 15u) : 0u;
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
            const float* vsm = reinterpret_cast<const float*>(v);
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
        const uint64_t polKeep = dev::policyEvictLast();
        unsigned char* xring = smem + L::kXOff + c * L::kXDepth * L::kXSlotBytes;
        const uint32_t xringA = dev::smemAddr(xring);
        const uint32_t laneX = t * L::kXRowStride + L::kLaneBytes * g; // this lane's bytes of row t
        bool ok = true;
        for (uint32_t s = 0; s < uint32_t(L::kPrefetch); ++s)
            ok = gatherRows<F, FPW, P>(smem, xring, barA, barU, packedX, cols, total, s, lane, c, polKeep, ok);
        uint32_t seq = 0;
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
                ok = gatherRows<F, FPW, P>(smem, xring, barA, barU, packedX, cols, total, seq + L::kPrefetch, lane, c,
                                        polKeep, ok);
                dev::cpAsyncWaitGroup<L::kPrefetch>();
                __syncwarp();
                const uint32_t stage = seq % L::kStages;
                if (ok && !boundedWait(barX + 8 * stage, (seq / L::kStages) & 1))
                    ok = false;
                if (!ok)
                    continue;
                const uint32_t stA = base + L::kStageOff + stage * L::kStageBytes;
                const uint32_t xsA = xringA + (seq & (L::kXDepth - 1)) * L::kXSlotBytes + laneX;
                const uint32_t inChunk = min(uint32_t(kChunk), panelCount - ch * kChunk);
#pragma unroll
                for (uint32_t pp = 0; pp < uint32_t(kChunk); ++pp) {
                    if (pp >= inChunk)
                        break;
                    const uint32_t m = dev::ldsU32(stA + L::kScaleBytes + L::kFragBytes + 4 * pp);
                    const uint4 s = dev::ldsV4(stA + 16 * (pp * 4 + t)); // (s_t, s_t, s_t+4, s_t+4)
                    const unsigned long long sa = (static_cast<unsigned long long>(s.y) << 32) | s.x;
                    const unsigned long long sb = (static_cast<unsigned long long>(s.w) << 32) | s.z;
                    const uint32_t rowA = xsA + pp * 8 * L::kXRowStride;
                    const uint32_t rowB = rowA + 4 * L::kXRowStride;
                    uint32_t da[L::kParts * 2], db[L::kParts * 2]; // dequantized sources t and t+4
                    if constexpr (L::kLaneBytes == 8) {
                        const uint2 wa = dev::ldsV2(rowA);
                        const uint2 wb = dev::ldsV2(rowB);
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
                        uint32_t t0[4];
                        dev::dequant4(dev::ldsU32(rowA), sa, t0);
                        da[0] = t0[0]; da[1] = t0[1]; da[2] = t0[2]; da[3] = t0[3];
                        dev::dequant4(dev::ldsU32(rowB), sb, t0);
                        db[0] = t0[0]; db[1] = t0[1]; db[2] = t0[2]; db[3] = t0[3];
                    }
                    const uint32_t fragA = stA + L::kScaleBytes + 8 * (pp * 4 * 32 + lane);
#pragma unroll
                    for (int rw = 0; rw < 4; ++rw) {
                        if (m & (1u << rw)) {
                            const uint2 bf = dev::ldsV2(fragA + 8 * 32 * rw);
#pragma unroll
                            for (int jj = 0; jj < L::kParts; ++jj)
                                dev::mmaTf32(acc[rw][jj], da[2 * jj], da[2 * jj + 1], db[2 * jj], db[2 * jj + 1], bf.x,
                                             bf.y);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0)
                    dev::mbarArrive(barE + 8 * stage);
            }
            // ---- write-back of this task ----
            if (task.sw == kSkipTask) // a padding entry: no panels, no rows
                continue;
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
                        const uint32_t r = e / kVec, vv = e % kVec;
                        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
                        for (uint32_t item = red.begin; item < red.end; ++item) {
                            const uint64_t blk = matrix.partialIds[item];
                            const float4 p = __ldcg(reinterpret_cast<const float4*>(partials + (blk * 8 + r) * F) + vv);
                            sum.x += p.x;
                            sum.y += p.y;
                            sum.z += p.z;
                            sum.w += p.w;
                        }
                        __stcs(reinterpret_cast<float4*>(output + uint64_t(row0 + r) * F) + vv, sum);
                    }
                }
            }
            namedBarrier(1, 32 * L::kConsumers); // flags[0] is reused by the next split task
        }
        dev::cpAsyncWaitAll();
        if (!ok)
            flags[1] = 1;
    }
    __syncthreads();
}

} // namespace
} // namespace tcc
