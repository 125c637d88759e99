// Tensor-memory SpMM kernel (tcgen05, sm_100a): the persistent sweep of
// spmm_persistent.cuh with the tile product moved to the 5th-generation tensor core.
//
// Per panel (8 source slots x the 32 rows of a window) and 128-feature slice the CTA issues ONE
//     tcgen05.mma.kind::tf32  D[128 features x 64] += A[128 x 8 sources] * B[8 x 64]
// with
//   A  the INT8 feature bytes of the 8 source rows as exact floats (X^T; every int8 is a TF32
//      value), written straight into tensor memory by the consumer warps (tcgen05.st);
//   B  the panel's values with the per-source scale folded in, b = tf32(a) * scale, as a dense
//      K-major tile in shared memory: columns 0-31 hold tf32(b) and columns 32-63 the TF32
//      remainder tf32(b - tf32(b)), so hi + lo carries b to 22 significant bits. A producer warp
//      builds it (zero fill plus a scatter of the panel's nonzeros);
//   D  the window's FP32 accumulator in tensor memory; Y row j = D[:, j] + D[:, 32 + j].
// Every product the tensor core forms is exact, so each term is q * tf32(a) * scale to 22 bits:
// within 2^-11 relative of the reference's tf32_rna(a) * tf32_rna(float(q) * scale)
// (src/kernel/spmm_kernel.cuh:7-19,45-57), half its stated bound; the scale multiply moves
// from 1024 feature values per panel to the panel's few nonzeros.
//
// Warp roles (the chunks - 4 panels, 32 source slots - of the CTA's tasks b, b+G, ... form one
// stream; producer pw owns chunks pw, pw+P, ... and every ring slot they map to):
//   consumers 0..F/32-1  warp w owns TMEM lane quarter w%4 of slice w/4 (32 features). X step
//                        (kPrefetch chunks ahead): cp.async of its 32 bytes of the chunk's 32
//                        packed source rows (L2 evict-last: rows are shared by neighbouring
//                        windows). Then it converts them to floats in the stage's A columns.
//   producers (P warps)  A step  (kALead ahead): bulk copies (TMA engine) of the chunk's 32
//                                source IDs and metadata words;
//                        V step  (kVLead ahead): cp.async of the value range and 32 scales;
//                        B step  the stage's B tiles (values times scales), then publish it.
//   MMA warp             one thread issues the MMAs of each chunk and the commits.
//
// Feature order inside a consumer's TMEM lane quarter: lane l holds feature
//     16 * (g / 4) + 2 * (g % 4) + {0, 8, 1, 9}[l / 8],   g = l % 8,
// which lets thread t fill its lanes from ONE 32-bit word (packed16 bytes 4(t/4)..4(t/4)+3) of
// each of two source rows. The epilogue undoes it (one 128-byte row segment per store).
//
// Synchronisation (all mbarrier waits bounded, about two seconds each):
//   aLand[a]  A step bulk copies -> all     : IDs and metadata of the chunk landed
//   aUsed[a]  consumers -> producer         : IDs read (X step issued), the slot may be refilled
//   vFull[v]  V step cp.async -> producer   : values and scales landed
//   bFull[s]  producer -> consumers         : B tiles of stage s written
//   aFull[s]  consumers -> MMA              : A columns of stage s stored (implies bFull[s])
//   sFree[s]  MMA commit -> producer        : the MMAs reading stage s are complete; the
//                                             producer's next bFull[s] passes this on to the
//                                             consumers (their A columns are free again)
//   dFull     MMA commit -> consumers       : the accumulator holds the window's result
//   dFree     consumers -> MMA              : the accumulator has been read (the next window's
//                                             first MMA overwrites it)
#pragma once
#include "spmm_persistent.cuh"

namespace tcc {
namespace {

template <int F, int STAGES, int P> struct Tmem {
    static constexpr int kSlices = F / 128;
    static constexpr int kConsumers = F / 32;
    static constexpr int kProducers = P;
    static constexpr int kProducerWarp = kConsumers;
    static constexpr int kMmaWarp = kConsumers + P;
    static constexpr int kThreads = 32 * (kConsumers + P + 1);
    static constexpr int kStages = STAGES;
    // Consumer X rings (one per consumer warp): 32 rows x 32 bytes per chunk, rows 48 bytes
    // apart so the word loads of two rows of a panel are bank-conflict free.
    static constexpr int kXDepth = 4;
    static constexpr int kPrefetch = kXDepth - 1;
    static constexpr int kXRowStride = 48;
    static constexpr int kXSlotBytes = 32 * kXRowStride;
    // Producer rings.
    static constexpr int kALead = 10, kARing = 16;
    static constexpr int kVLead = 5, kVRing = 8;
    static constexpr int kVCap = 128;
    static constexpr int kASlotBytes = 128 + 256 + 16; // ids, metadata, header (p0, np)
    static constexpr int kVSlotBytes = kVCap * 4 + 128; // values, scales
    // Stage: four B tiles (one per panel, 64 columns x 8 sources TF32, K-major core matrices:
    // element (column n, source k) at (n%8)*16 + (n/8)*256 + (k/4)*128 + (k%4)*4).
    static constexpr int kBTileBytes = 2048;
    static constexpr int kBOff = 0;
    static constexpr int kXOff = kBOff + kStages * kChunk * kBTileBytes;
    static constexpr int kAOff = kXOff + kConsumers * kXDepth * kXSlotBytes;
    static constexpr int kVOff = kAOff + kARing * kASlotBytes;
    static constexpr int kVBaseOff = kVOff + kVRing * kVSlotBytes;
    static constexpr int kFlagOff = kVBaseOff + 32;
    static constexpr int kBarOff = kFlagOff + 16;
    // bFull, aFull, sFree [kStages]; dFull, dFree (two words reserved each); aLand, aUsed
    // [kARing]; vFull [kVRing]; drain
    static constexpr int kBars = 3 * kStages + 4 + 2 * kARing + kVRing + 1;
    static constexpr int kBytes = kBarOff + 8 * kBars;
    // Tensor memory: per slice, kStages A slots of 32 columns (4 panels x 8 sources) and the
    // accumulator of 64 columns (hi and lo products of the window's 32 rows); allocation is a
    // power of two.
    static constexpr int kSliceCols = 32 * kStages + 64;
    static constexpr int kColsUsed = kSlices * kSliceCols;
    static constexpr int kTmemCols = kColsUsed <= 32    ? 32
                                     : kColsUsed <= 64  ? 64
                                     : kColsUsed <= 128 ? 128
                                     : kColsUsed <= 256 ? 256
                                                        : 512;
    static constexpr int kMaxCtasPerSm = 512 / kTmemCols;
    static_assert(kColsUsed <= 512, "tensor memory");
    static_assert(kVRing <= 8 && kARing >= kALead + 2 && kVRing > kVLead && kALead > kVLead && kPrefetch <= kALead,
                  "rings");
    static_assert(kARing % P == 0 && kVRing % P == 0 && kStages % P == 0, "every ring slot has one producer");
    static_assert((kARing & (kARing - 1)) == 0 && (kVRing & (kVRing - 1)) == 0 && (kStages & (kStages - 1)) == 0 &&
                      (kXDepth & (kXDepth - 1)) == 0,
                  "power-of-two rings");
    static_assert(kXOff % 16 == 0 && kAOff % 16 == 0 && kVOff % 16 == 0 && kBarOff % 8 == 0, "alignment");
    // Instruction descriptor: D FP32 (bits 4-5 = 1), A and B TF32 (bits 7-9, 10-12 = 2), both
    // K-major, N = 64 (bits 17-22 = N/8), M = 128 (bits 24-28 = M/16).
    static constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
};

// Shared-memory matrix descriptor of one B tile (no swizzle, K-major core matrices of 8 rows
// x 16 bytes): start address >> 4, leading (K) byte offset 128 >> 4, stride (8-row group) byte
// offset 256 >> 4, descriptor version 1 (bits 46-47).
__device__ __forceinline__ unsigned long long bTileDesc(uint32_t smemAddr) {
    return static_cast<unsigned long long>((smemAddr >> 4) & 0x3FFFu) | (static_cast<unsigned long long>(128 >> 4) << 16) |
           (static_cast<unsigned long long>(256 >> 4) << 32) | (1ull << 46);
}

// TMEM lane (0..31 within a consumer's quarter) -> feature within the consumer's 32.
__device__ __forceinline__ int tmemLaneFeature(int l) {
    const int g = l & 7, part = l >> 3;
    return 16 * (g >> 2) + 2 * (g & 3) + ((part & 1) << 3) + (part >> 1);
}

// Consumer X step of chunk s: warp w gathers bytes 32w..32w+31 of the chunk's 32 packed source
// rows (two 16-byte cp.async per row, invalid slots zero-filled) as one cp.async group, then
// (barUsed != 0) tells the producer that the chunk's IDs have been read. Returns false when the
// wait ran out. L is the kernel's shared-memory layout.
template <typename L, int F>
__device__ __forceinline__ bool gatherSlice(unsigned char* smem, uint32_t xring, uint32_t barLand, uint32_t barUsed,
                                            const int8_t* __restrict__ packedX, uint32_t cols, uint32_t total,
                                            uint32_t s, int lane, int w, uint64_t policy, bool ok) {
    if (ok && s < total) {
        const uint32_t aslot = s % L::kARing;
        if (!boundedWait(barLand + 8 * aslot, (s / L::kARing) & 1)) {
            ok = false;
        } else {
            const unsigned char* a = smem + L::kAOff + aslot * L::kASlotBytes;
            const uint32_t np = reinterpret_cast<const uint32_t*>(a + 384)[1];
            const uint32_t dst = xring + (s % L::kXDepth) * L::kXSlotBytes;
#pragma unroll
            for (int pass = 0; pass < 2; ++pass) {
                const int row = pass * 16 + (lane >> 1), piece = lane & 1;
                const uint32_t id = uint32_t(row >> 3) < np ? reinterpret_cast<const uint32_t*>(a)[row] : 0xFFFFFFFFu;
                const bool valid = id < cols;
                dev::cpAsync16Hint(dst + row * L::kXRowStride + 16 * piece,
                                   valid ? static_cast<const void*>(packedX + uint64_t(id) * F + 32 * w + 16 * piece)
                                         : static_cast<const void*>(packedX),
                                   valid ? 16u : 0u, policy);
            }
            __syncwarp();
            if (lane == 0 && barUsed != 0)
                dev::mbarArrive(barUsed + 8 * aslot);
        }
    }
    dev::cpAsyncCommit();
    return ok;
}

template <int F, int STAGES, int P>
__global__ void __launch_bounds__(Tmem<F, STAGES, P>::kThreads, Tmem<F, STAGES, P>::kMaxCtasPerSm)
    spmmTmemKernel(const tcc_sw32_device_view matrix, const int8_t* __restrict__ packedX,
                   const float* __restrict__ scales, float* __restrict__ output, uint32_t rows, uint32_t cols,
                   float* __restrict__ partials, uint32_t* __restrict__ counters) {
    using L = Tmem<F, STAGES, P>;
    extern __shared__ __align__(128) unsigned char smem[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t base = dev::smemAddr(smem);
    const uint32_t barB = base + L::kBarOff;        // bFull [kStages]
    const uint32_t barA = barB + 8 * L::kStages;    // aFull [kStages]
    const uint32_t barS = barA + 8 * L::kStages;    // sFree [kStages]
    const uint32_t barD = barS + 8 * L::kStages;    // dFull [2]
    const uint32_t barR = barD + 16;                // dFree [2]
    const uint32_t barL = barR + 16;                // aLand [kARing]
    const uint32_t barU = barL + 8 * L::kARing;     // aUsed [kARing]
    const uint32_t barV = barU + 8 * L::kARing;     // vFull [kVRing]
    const uint32_t barF = barV + 8 * L::kVRing;     // drain
    volatile uint32_t* flags = reinterpret_cast<volatile uint32_t*>(smem + L::kFlagOff);
    if (threadIdx.x == 0) {
        for (int s = 0; s < L::kStages; ++s) {
            dev::mbarInit(barB + 8 * s, 1);
            dev::mbarInit(barA + 8 * s, L::kConsumers);
            dev::mbarInit(barS + 8 * s, 1);
        }
        for (int d = 0; d < 2; ++d) {
            dev::mbarInit(barD + 8 * d, 1);
            dev::mbarInit(barR + 8 * d, L::kConsumers);
        }
        for (int s = 0; s < L::kARing; ++s) {
            dev::mbarInit(barL + 8 * s, 1);
            dev::mbarInit(barU + 8 * s, L::kConsumers);
        }
        for (int s = 0; s < L::kVRing; ++s)
            dev::mbarInit(barV + 8 * s, 32);
        dev::mbarInit(barF, 1);
        flags[0] = flags[1] = flags[3] = 0; // flags[2] receives the TMEM address (allocating warp)
        dev::fenceBarrierInit();
    }
    if (warp == L::kMmaWarp) {
        dev::tmemAlloc(base + L::kFlagOff + 8, L::kTmemCols);
        dev::tmemRelinquish();
    }
    dev::tcFenceBefore();
    __syncthreads();
    dev::tcFenceAfter();
    const uint32_t tmem = flags[2];
    const uint32_t total = ctaChunkCount(matrix, lane);

    if (warp >= L::kProducerWarp && warp < L::kMmaWarp) {
        // =================================== producers ====================================
        const uint64_t polStream = dev::policyEvictFirst();
        const uint64_t polKeep = dev::policyEvictLast();
        uint32_t* vBase = reinterpret_cast<uint32_t*>(smem + L::kVBaseOff);
        const int pp = lane >> 3, k = lane & 7;
        const uint32_t pw = warp - L::kProducerWarp;
        ChunkWalker walk;
        walk.start(matrix);
        for (uint32_t i = 0; i < pw; ++i)
            walk.advance(matrix);
        uint32_t seqA = pw, seqV = pw;
        bool ok = true;
        for (uint32_t seqF = pw; seqF < total && ok; seqF += P) {
            // ---- A steps: IDs and metadata of chunks up to seqF + kALead (one lane) ----
            for (; seqA < total && seqA <= seqF + L::kALead; seqA += P) {
                const uint32_t slot = seqA % L::kARing;
                if (seqA >= uint32_t(L::kARing) && !boundedWait(barU + 8 * slot, ((seqA / L::kARing) - 1) & 1)) {
                    ok = false;
                    break;
                }
                const uint32_t p0 = walk.next;
                const uint32_t np = min(uint32_t(kChunk), walk.end - p0);
                if (lane == 0) {
                    const uint32_t a = base + L::kAOff + slot * L::kASlotBytes;
                    uint32_t* header = reinterpret_cast<uint32_t*>(smem + L::kAOff + slot * L::kASlotBytes + 384);
                    header[0] = p0;
                    header[1] = np;
                    dev::fenceProxyAsyncShared(); // earlier generic reads of the slot before the copies
                    dev::mbarArriveExpectTx(barL + 8 * slot, 96 * np);
                    dev::bulkCopyG2SHint(a, matrix.sourceIds + uint64_t(p0) * 8, 32 * np, barL + 8 * slot, polStream);
                    dev::bulkCopyG2SHint(a + 128, matrix.sourceMetadata + uint64_t(p0) * 8, 64 * np, barL + 8 * slot,
                                         polStream);
                }
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
                if (!boundedWait(barL + 8 * aslot, (seqV / L::kARing) & 1)) {
                    ok = false;
                    break;
                }
                const unsigned char* a = smem + L::kAOff + aslot * L::kASlotBytes;
                unsigned char* v = smem + L::kVOff + vslot * L::kVSlotBytes;
                const uint32_t np = reinterpret_cast<const uint32_t*>(a + 384)[1];
                const bool inRange = uint32_t(pp) < np;
                const uint32_t id = inRange ? *reinterpret_cast<const uint32_t*>(a + 4 * lane) : 0xFFFFFFFFu;
                const uint64_t meta = inRange ? *reinterpret_cast<const uint64_t*>(a + 128 + 8 * lane) : 0ull;
                const bool valid = id < cols;
                dev::cpAsync4Hint(dev::smemAddr(v + 4 * L::kVCap + 4 * lane),
                                  valid ? static_cast<const void*>(scales + id) : static_cast<const void*>(scales),
                                  valid ? 4u : 0u, polKeep);
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
            // ---- B step: B tiles of chunk seqF; publish the stage ----
            const uint32_t aslot = seqF % L::kARing, vslot = seqF % L::kVRing, stage = seqF % L::kStages;
            if (!boundedWait(barV + 8 * vslot, (seqF / L::kVRing) & 1) ||
                (seqF >= uint32_t(L::kStages) &&
                 !boundedWaitBackoff(barS + 8 * stage, ((seqF / L::kStages) - 1) & 1))) {
                ok = false;
                break;
            }
            const unsigned char* a = smem + L::kAOff + aslot * L::kASlotBytes;
            const unsigned char* v = smem + L::kVOff + vslot * L::kVSlotBytes;
            const uint32_t np = reinterpret_cast<const uint32_t*>(a + 384)[1];
            unsigned char* tiles = smem + L::kBOff + stage * (kChunk * L::kBTileBytes);
            const float scale = reinterpret_cast<const float*>(v + 4 * L::kVCap)[lane];
            {
                uint4* z = reinterpret_cast<uint4*>(tiles);
#pragma unroll
                for (int i = 0; i < kChunk * L::kBTileBytes / 16 / 32; ++i)
                    z[i * 32 + lane] = make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
            const uint64_t meta = uint32_t(pp) < np ? *reinterpret_cast<const uint64_t*>(a + 128 + 8 * lane) : 0ull;
            uint32_t mask = static_cast<uint32_t>(meta);
            const uint32_t first = static_cast<uint32_t>(meta >> 32);
            const uint32_t vb = vBase[vslot];
            const float* vsm = reinterpret_cast<const float*>(v);
            uint32_t* tile = reinterpret_cast<uint32_t*>(tiles + pp * L::kBTileBytes + (k >> 2) * 128 + (k & 3) * 4);
            uint32_t j = 0;
            while (mask) {
                const int r = __ffs(mask) - 1;
                mask &= mask - 1;
                const float value = vb != 0xFFFFFFFFu ? vsm[first + j - vb] : __ldg(matrix.values + first + j);
                ++j;
                // b = tf32(a) * scale as a TF32 pair hi + lo (22 significant bits): rows 0-31
                // of the tile hold hi, rows 32-63 lo.
                const float b = __uint_as_float(dev::tf32Exact(value)) * scale;
                const uint32_t hi = dev::tf32Exact(b);
                const uint32_t lo = dev::tf32Exact(b - __uint_as_float(hi));
                tile[((r & 7) * 16 + (r >> 3) * 256) / 4] = hi;
                tile[((r & 7) * 16 + (r >> 3) * 256 + 1024) / 4] = lo;
            }
            dev::fenceProxyAsyncShared();
            __syncwarp();
            if (lane == 0)
                dev::mbarArrive(barB + 8 * stage);
        }
        if (!ok)
            flags[1] = 1;
        dev::cpAsyncWaitAll();
        // No bulk copy may still be writing into this CTA's shared memory at exit (after a
        // wait ran out, a filled slot may not have been waited for).
        for (uint32_t s = seqA >= L::kARing + pw ? seqA - L::kARing : pw; s < seqA; s += P)
            boundedWait(barL + 8 * (s % L::kARing), (s / L::kARing) & 1);
    } else if (warp == L::kMmaWarp) {
        // ================================ MMA issuer (one thread) =========================
        if (lane == 0) {
            bool ok = true, issued = false;
            uint32_t seq = 0, windows = 0;
            for (uint64_t tk = blockIdx.x; tk < matrix.taskCount; tk += gridDim.x) {
                const tcc_sw32_task task = matrix.tasks[tk];
                const uint32_t panelCount = task.end - task.begin;
                if (panelCount == 0)
                    continue;
                // One accumulator (64 columns): the window's first MMA overwrites it once the
                // consumers have read the previous window's result.
                if (ok && windows >= 1 && !boundedWaitBackoff(barR, (windows - 1) & 1))
                    ok = false;
                ++windows;
                dev::tcFenceAfter();
                const uint32_t nch = (panelCount + kChunk - 1) / kChunk;
                for (uint32_t ch = 0; ch < nch; ++ch, ++seq) {
                    // aFull[stage] follows bFull[stage]: every consumer waited for it first.
                    const uint32_t stage = seq % L::kStages;
                    if (ok && !boundedWaitBackoff(barA + 8 * stage, (seq / L::kStages) & 1))
                        ok = false;
                    if (!ok)
                        continue;
                    dev::tcFenceAfter();
                    const uint32_t inChunk = min(uint32_t(kChunk), panelCount - ch * kChunk);
                    const uint32_t tiles = base + L::kBOff + stage * (kChunk * L::kBTileBytes);
                    for (uint32_t pp = 0; pp < inChunk; ++pp) {
                        const unsigned long long desc = bTileDesc(tiles + pp * L::kBTileBytes);
#pragma unroll
                        for (int sl = 0; sl < L::kSlices; ++sl)
                            dev::mmaTf32Ts(tmem + sl * L::kSliceCols + 32 * L::kStages,
                                           tmem + sl * L::kSliceCols + 32 * stage + 8 * pp, desc, L::kIdesc,
                                           (ch | pp) != 0);
                    }
                    issued = true;
                    dev::tcCommit(barS + 8 * stage);
                }
                if (ok)
                    dev::tcCommit(barD);
            }
            if (issued) { // every MMA is complete before the tensor memory is released
                dev::tcCommit(barF);
                if (!boundedWait(barF, 0))
                    ok = false;
            }
            if (!ok)
                flags[1] = 1;
        }
        __syncwarp();
    } else {
        // ==================================== consumers ===================================
        const int quarter = warp & 3, slice = warp >> 2;
        const int g = lane >> 2, c = lane & 3;
        const uint64_t polKeep = dev::policyEvictLast();
        const uint32_t xring = base + L::kXOff + warp * L::kXDepth * L::kXSlotBytes;
        const uint32_t tLane = uint32_t(32 * quarter) << 16;
        const uint32_t aTmem = tmem + slice * L::kSliceCols + tLane;
        const uint32_t dTmem = tmem + slice * L::kSliceCols + 32 * L::kStages + tLane;
        const uint32_t feature = slice * 128 + 32 * quarter + tmemLaneFeature(lane);
        const uint32_t xLane = xring + 4 * g + 2 * c * L::kXRowStride;
        bool ok = true;
        for (uint32_t s = 0; s < uint32_t(L::kPrefetch); ++s)
            ok = gatherSlice<L, F>(smem, xring, barL, barU, packedX, cols, total, s, lane, warp, polKeep, ok);
        uint32_t seq = 0, windows = 0;
        tcc_sw32_task nextTask{};
        if (blockIdx.x < matrix.taskCount)
            nextTask = matrix.tasks[blockIdx.x];
        for (uint64_t tk = blockIdx.x; tk < matrix.taskCount; tk += gridDim.x) {
            const tcc_sw32_task task = nextTask;
            if (tk + gridDim.x < matrix.taskCount)
                nextTask = matrix.tasks[tk + gridDim.x];
            const uint32_t panelCount = task.end - task.begin;
            const uint32_t nch = (panelCount + kChunk - 1) / kChunk;
            for (uint32_t ch = 0; ch < nch; ++ch, ++seq) {
                ok = gatherSlice<L, F>(smem, xring, barL, barU, packedX, cols, total, seq + L::kPrefetch, lane, warp,
                                       polKeep, ok);
                dev::cpAsyncWaitGroup<L::kPrefetch>();
                __syncwarp();
                // bFull[stage] also tells that the MMAs of chunk seq - kStages are complete
                // (the producer waited for them), so the stage's A columns may be rewritten.
                const uint32_t stage = seq % L::kStages;
                if (ok && !boundedWait(barB + 8 * stage, (seq / L::kStages) & 1))
                    ok = false;
                if (!ok)
                    continue;
                dev::tcFenceAfter();
                const uint32_t xs = xLane + (seq & (L::kXDepth - 1)) * L::kXSlotBytes;
                uint32_t lo[16], hi[16];
#pragma unroll
                for (int pp = 0; pp < kChunk; ++pp) {
                    const uint32_t wa = dev::ldsU32(xs + 8 * pp * L::kXRowStride) ^ 0x80808080u;
                    const uint32_t wb = dev::ldsU32(xs + (8 * pp + 1) * L::kXRowStride) ^ 0x80808080u;
                    dev::int8PairToFloat<0>(wa, wb, lo[4 * pp + 0], lo[4 * pp + 1]);
                    dev::int8PairToFloat<1>(wa, wb, lo[4 * pp + 2], lo[4 * pp + 3]);
                    dev::int8PairToFloat<2>(wa, wb, hi[4 * pp + 0], hi[4 * pp + 1]);
                    dev::int8PairToFloat<3>(wa, wb, hi[4 * pp + 2], hi[4 * pp + 3]);
                }
                dev::tcStore16x256bx4(aTmem + 32 * stage, lo);
                dev::tcStore16x256bx4(aTmem + 32 * stage + (16u << 16), hi);
                dev::tcWaitSt();
                dev::tcFenceBefore();
                __syncwarp();
                if (lane == 0)
                    dev::mbarArrive(barA + 8 * stage);
            }
            // ---- epilogue of this window ----
            const uint32_t rowBase = task.sw * 32;
            const bool split = task.partial != kNoPartial;
            const bool haveWs = !split || (partials != nullptr && counters != nullptr);
            if (!haveWs && threadIdx.x == 0)
                atomicOr(&gDeviceStatus, 2u);
            bool loaded = false;
            if (panelCount > 0) {
                if (ok && !boundedWait(barD, windows & 1))
                    ok = false;
                ++windows;
                loaded = ok;
                if (loaded)
                    dev::tcFenceAfter();
            }
            // Y row j = column j (the hi products) + column 32 + j (the lo products), stored 16
            // rows at a time: straight to Y, or to the split task's partial block of the row's
            // 8-row group.
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t h[16], l[16];
                if (loaded) {
                    dev::tcLoad32x32bx16(dTmem + 16 * half, h);
                    dev::tcLoad32x32bx16(dTmem + 32 + 16 * half, l);
                    dev::tcWaitLd();
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        h[j] = l[j] = 0u;
                }
                if (!haveWs)
                    continue;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int row = 16 * half + j;
                    const float y = __uint_as_float(h[j]) + __uint_as_float(l[j]);
                    if (!split) {
                        if (rowBase + row < rows)
                            __stcs(output + uint64_t(rowBase + row) * F + feature, y);
                    } else if (task.mask & (1u << (row >> 3))) {
                        const uint64_t block = task.partial + __popc(task.mask & ((1u << (row >> 3)) - 1));
                        __stcg(partials + (block * 8 + (row & 7)) * F + feature, y);
                    }
                }
            }
            if (panelCount > 0) {
                if (loaded)
                    dev::tcFenceBefore();
                __syncwarp();
                if (lane == 0)
                    dev::mbarArrive(barR);
            }
            if (!split || !haveWs)
                continue;
            // Last-arriver merge among the consumer warps (reference src/kernel/spmm_kernel.cuh:250-282).
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
    dev::tcFenceBefore();
    __syncthreads();
    dev::tcFenceAfter();
    if (warp == L::kMmaWarp)
        dev::tmemDealloc(tmem, L::kTmemCols);
}

} // namespace
} // namespace tcc
