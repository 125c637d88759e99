// Tensor-memory SpMM kernel (tcgen05, sm_100a): the fast path of launchSpmmInt8.
//
// Per panel (8 source slots x the 32 rows of a window) and 128-feature slice one thread issues
//     tcgen05.mma.cta_group::1.kind::tf32  D[128 features x 64] += A[128 x 8 sources] * B[8 x 64]
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
// from the 1024 feature values of a panel to its few nonzeros.
//
// The kernel is persistent: CTA b of a grid of G takes tasks b, b+G, b+2G, ... and the chunks
// (8 panels = 64 source slots) of those tasks form one stream. Tensor memory holds one A stage
// of 64 columns and the 64-column accumulator (128 columns, 4 CTAs per SM at F = 128), shared
// memory one buffer of B tiles, so the stage is refilled only after the MMAs of chunk c are
// complete. The producer (B tiles) and the consumers (A columns) then refill it at the same
// time, both waiting on that commit, and the MMA thread waits for both. The other CTAs of the
// SM fill the gap.
//
// Feature order inside a consumer's TMEM lane quarter: lane l holds feature
//     16 * (g / 4) + 2 * (g % 4) + {0, 8, 1, 9}[l / 8],   g = l % 8,
// which lets thread t fill its lanes from ONE 32-bit word (packed16 bytes 4(t/4)..4(t/4)+3) of
// each of two source rows. The epilogue undoes it (one 128-byte row segment per store).
//
// Roles (chunks of the CTA's tasks b, b+G, ... form one stream; producer pw owns chunks pw,
// pw+P, ...):
//   producers (P warps)  A step (bulk copies of the chunk's 64 IDs and metadata words, kALead
//                        chunks ahead), V step (kVLead ahead: one bulk copy of the value range,
//                        cp.async of the 64 scales and of the chunk's 64 whole source rows into the
//                        shared X ring, 16 bytes per lane, F / 16 lanes per row), B step (the
//                        chunk's 8 B tiles in the one shared-memory B buffer).
//   consumers 0..F/32-1  warp w owns TMEM lane quarter w%4 of slice w/4 (32 features): it reads its
//                        32 bytes of the chunk's rows from the X ring and stores the A columns. It
//                        touches no global memory in the chunk loop.
//   MMA warp             runs the issue loop as a warp; one elected lane issues the chunk's MMAs and
//                        the commits.
// The X ring keeps rows at a stride of F + 16 bytes, so the rows 2c and 2c + 1 that lane group c
// reads fall in distinct banks. Gathering whole rows in the producers instead of 32-byte quarters
// in each consumer took about 1,000 cycles per chunk off the consumers, the critical role, and
// made a warp-wide copy touch 4 lines instead of 16.
// Synchronisation: bFull (producer -> MMA: B tiles written), aFull (consumers -> MMA: A columns
// stored), sFree[c % 2] (MMA commit of chunk c -> the producer and the consumers of chunk c + 1,
// who then refill the B tiles and the A columns at the same time), dFull/dFree for the
// accumulator, aLand and vFull for the producer rings, xFull (the owning producer's copies of a
// chunk's rows have landed) and xFree (consumers -> producers: the X slot may be refilled). A
// slots are read only by the producer that fills them. All waits bounded.
// Every copy uses the default L2 policy: evict-last on X and evict-first on the format arrays
// cost 3%. Invalid slots issue no copy at all: their A columns keep stale (finite) bytes, which
// meet all-zero rows of B, and the producer skips their scales.
#pragma once
#include "spmm_persistent.cuh"

namespace tcc {
namespace {

constexpr int kChunk8 = 8; // panels per chunk: 64 source slots, two per producer lane
constexpr uint32_t kTestStallOddCtas = 1; // testFlags bit: stall the MMA thread of odd CTAs

// Instruction descriptor of the MMA: D FP32 (bits 4-5 = 1), A and B TF32 (bits 7-9, 10-12 =
// 2), both K-major, N = 64 (bits 17-22 = N/8), M = 128 (bits 24-28 = M/16).
constexpr uint32_t kIdescTf32M128N64 =
    (1u << 4) | (2u << 7) | (2u << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);

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

template <int F, int P> struct Tmem8 {
    static constexpr int kSlices = F / 128;
    static constexpr int kConsumers = F / 32;
    static constexpr int kProducers = P;
    static constexpr int kProducerWarp = kConsumers;
    static constexpr int kMmaWarp = kConsumers + P;
    static constexpr int kThreads = 32 * (kConsumers + P + 1);
    static constexpr int kSlots = 8 * kChunk8;
    // X ring, shared by the consumers: kXDepth chunks of 64 whole packed source rows. Row r of a
    // chunk sits at r * (F + 16): the 16-byte pad puts rows 2c and 2c + 1, which lane group c
    // reads, in distinct banks. The producer that owns a chunk copies its rows (kLanesPerRow
    // lanes of 16 bytes per row, kRowsPerCopy rows per warp-wide cp.async).
    static constexpr int kXDepth = 3;
    static constexpr int kXRowStride = F + 16;
    static constexpr int kXSlotBytes = kSlots * kXRowStride;
    static constexpr int kLanesPerRow = F / 16;
    static constexpr int kRowsPerCopy = 32 / kLanesPerRow;
    // Producer rings.
    static constexpr int kALead = 5, kARing = 8;
    static constexpr int kVLead = 2, kVRing = 4;
    static constexpr int kVCap = 256;
    static constexpr int kHeaderOff = 4 * kSlots + 8 * kSlots;  // after ids and metadata
    static constexpr int kASlotBytes = kHeaderOff + 16;
    static constexpr int kVSlotBytes = kVCap * 4 + 4 * kSlots; // values, scales
    static constexpr int kBTileBytes = 2048;
    static constexpr int kBOff = 0;
    static constexpr int kXOff = kBOff + kChunk8 * kBTileBytes;
    static constexpr int kAOff = kXOff + kXDepth * kXSlotBytes;
    static constexpr int kVOff = kAOff + kARing * kASlotBytes;
    static constexpr int kVBaseOff = kVOff + kVRing * kVSlotBytes;
    static constexpr int kFlagOff = kVBaseOff + 32;
    static constexpr int kBarOff = kFlagOff + 16;
    // bFull, aFull, sFree [2] (by chunk parity); dFull, dFree (two words reserved each); aLand
    // [kARing]; vFull [kVRing]; xFull, xFree [kXDepth]; drain
    static constexpr int kBars = 4 + 4 + kARing + kVRing + 2 * kXDepth + 1;
    static constexpr int kBytes = kBarOff + 8 * kBars;
    // Tensor memory per slice: the A stage (64 columns: 8 panels x 8 sources) and the
    // accumulator (64 columns).
    static constexpr int kSliceCols = 8 * kChunk8 + 64;
    static constexpr int kColsUsed = kSlices * kSliceCols;
    static constexpr int kTmemCols = kColsUsed <= 128 ? 128 : kColsUsed <= 256 ? 256 : 512;
    static constexpr int kMaxCtasPerSm = 512 / kTmemCols;
    static_assert(kColsUsed <= 512, "tensor memory");
    static_assert(kVRing <= 8 && kARing >= kALead + 2 && kVRing > kVLead && kALead > kVLead && kXDepth > kVLead,
                  "rings");
    static_assert(kXRowStride % 16 == 0 && (kXRowStride / 2) % 32 == 8 && kSlots % kRowsPerCopy == 0,
                  "X rows: 16-byte aligned, conflict-free reads");
    static_assert(kARing % P == 0 && kVRing % P == 0, "every ring slot has one producer");
    static_assert(P == 1 || P == 2, "sFree[c % 2] gives each producer consecutive phases only for P <= 2");
    static_assert(kASlotBytes % 16 == 0 && kXOff % 16 == 0 && kAOff % 16 == 0 && kVOff % 16 == 0 && kBarOff % 8 == 0,
                  "alignment");
    static constexpr uint32_t kIdesc = kIdescTf32M128N64;
};

template <int F, int P>
__global__ void __launch_bounds__(Tmem8<F, P>::kThreads, Tmem8<F, P>::kMaxCtasPerSm)
    spmmTmem8Kernel(const tcc_sw32_device_view matrix, const int8_t* __restrict__ packedX,
                    const float* __restrict__ scales, float* __restrict__ output, uint32_t rows, uint32_t cols,
                    float* __restrict__ partials, uint32_t* __restrict__ counters, uint32_t testFlags) {
    using L = Tmem8<F, P>;
    extern __shared__ __align__(128) unsigned char smem[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t base = dev::smemAddr(smem);
    const uint32_t barB = base + L::kBarOff;   // bFull
    const uint32_t barA = barB + 8;            // aFull
    const uint32_t barS = barA + 8;            // sFree [2]
    const uint32_t barD = barS + 16;           // dFull [2]
    const uint32_t barR = barD + 16;           // dFree [2]
    const uint32_t barL = barR + 16;           // aLand [kARing]
    const uint32_t barV = barL + 8 * L::kARing;    // vFull [kVRing]
    const uint32_t barXF = barV + 8 * L::kVRing;   // xFull [kXDepth]
    const uint32_t barXE = barXF + 8 * L::kXDepth; // xFree [kXDepth]
    const uint32_t barF = barXE + 8 * L::kXDepth;  // drain
    volatile uint32_t* flags = reinterpret_cast<volatile uint32_t*>(smem + L::kFlagOff);
    if (threadIdx.x == 0) {
        dev::mbarInit(barB, 1);
        dev::mbarInit(barA, L::kConsumers);
        dev::mbarInit(barS, 1);
        dev::mbarInit(barS + 8, 1);
        for (int d = 0; d < 2; ++d) {
            dev::mbarInit(barD + 8 * d, 1);
            dev::mbarInit(barR + 8 * d, L::kConsumers);
        }
        for (int s = 0; s < L::kARing; ++s) {
            dev::mbarInit(barL + 8 * s, 1);
        }
        for (int s = 0; s < L::kVRing; ++s)
            dev::mbarInit(barV + 8 * s, 33); // the lanes' scale copies and lane 0's value-range copy
        for (int s = 0; s < L::kXDepth; ++s) {
            dev::mbarInit(barXF + 8 * s, 32); // the owning producer's lanes, once their copies land
            dev::mbarInit(barXE + 8 * s, L::kConsumers);
        }
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
    const uint32_t total = ctaChunkCountT<kChunk8>(matrix, lane);

    if (warp >= L::kProducerWarp && warp < L::kMmaWarp) {
        // =================================== producers ====================================
        uint32_t* vBase = reinterpret_cast<uint32_t*>(smem + L::kVBaseOff);
        const uint32_t pw = warp - L::kProducerWarp;
        ChunkWalkerT<kChunk8> walk;
        walk.start(matrix);
        for (uint32_t i = 0; i < pw; ++i)
            walk.advance(matrix);
        uint32_t seqA = pw, seqV = pw;
        bool ok = true;
        for (uint32_t seqF = pw; seqF < total && ok; seqF += P) {
            // ---- A steps: IDs and metadata of chunks up to seqF + kALead (one lane) ----
            for (; seqA < total && seqA <= seqF + L::kALead; seqA += P) {
                // The slot's previous chunk, seqA - kARing, belongs to this producer too (kARing is a
                // multiple of P), and its V and B steps are done: no other role reads A slots.
                const uint32_t slot = seqA % L::kARing;
                const uint32_t p0 = walk.next;
                const uint32_t np = min(uint32_t(kChunk8), walk.end - p0);
                if (lane == 0) {
                    const uint32_t a = base + L::kAOff + slot * L::kASlotBytes;
                    uint32_t* header =
                        reinterpret_cast<uint32_t*>(smem + L::kAOff + slot * L::kASlotBytes + L::kHeaderOff);
                    header[0] = p0;
                    header[1] = np;
                    dev::fenceProxyAsyncShared(); // earlier generic reads of the slot before the copies
                    dev::mbarArriveExpectTx(barL + 8 * slot, 96 * np);
                    dev::bulkCopyG2S(a, matrix.sourceIds + uint64_t(p0) * 8, 32 * np, barL + 8 * slot);
                    dev::bulkCopyG2S(a + 4 * L::kSlots, matrix.sourceMetadata + uint64_t(p0) * 8, 64 * np,
                                     barL + 8 * slot);
                }
#pragma unroll
                for (int i = 0; i < P; ++i)
                    walk.advance(matrix);
            }
            if (!ok)
                break;
            __syncwarp();
            // ---- V steps: value ranges, scales and X rows of chunks up to seqF + kVLead; the X
            // rows of chunk s go to X slot s % kXDepth once the consumers have released chunk
            // s - kXDepth from it ----
            for (; seqV < seqA && seqV <= seqF + L::kVLead; seqV += P) {
                const uint32_t aslot = seqV % L::kARing, vslot = seqV % L::kVRing, xslot = seqV % L::kXDepth;
                if (!boundedWait(barL + 8 * aslot, (seqV / L::kARing) & 1) ||
                    (seqV >= uint32_t(L::kXDepth) &&
                     !boundedWait(barXE + 8 * xslot, ((seqV / L::kXDepth) - 1) & 1))) {
                    ok = false;
                    break;
                }
                unsigned char* a = smem + L::kAOff + aslot * L::kASlotBytes;
                unsigned char* v = smem + L::kVOff + vslot * L::kVSlotBytes;
                const uint32_t np = reinterpret_cast<const uint32_t*>(a + L::kHeaderOff)[1];
                uint32_t lo = 0xFFFFFFFFu, hi = 0u;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t slot = lane + 32 * h;
                    const bool inRange = (slot >> 3) < np;
                    const uint32_t id = inRange ? reinterpret_cast<const uint32_t*>(a)[slot] : 0xFFFFFFFFu;
                    if (!inRange) // past the chunk's last panel: stale, marked invalid for the row copies
                        reinterpret_cast<uint32_t*>(a)[slot] = 0xFFFFFFFFu;
                    const uint64_t meta =
                        inRange ? reinterpret_cast<const uint64_t*>(a + 4 * L::kSlots)[slot] : 0ull;
                    // an invalid slot's scale is never read (its row mask is empty)
                    dev::cpAsync4If(dev::smemAddr(v + 4 * L::kVCap + 4 * slot), scales + id, id, cols);
                    const uint32_t mask = static_cast<uint32_t>(meta);
                    const uint32_t first = static_cast<uint32_t>(meta >> 32);
                    if (mask) {
                        lo = min(lo, first);
                        hi = max(hi, first + __popc(mask));
                    }
                }
                lo = __reduce_min_sync(0xFFFFFFFFu, lo);
                hi = __reduce_max_sync(0xFFFFFFFFu, hi);
                // The value range [lo, hi) from the 16-byte boundary at or below lo: its whole
                // 16-byte groups as one bulk copy, the last 0-3 values (which never reach past hi,
                // the end of the chunk's values) by cp.async.
                const uint32_t lo4 = lo & ~3u;
                const uint32_t span = hi > lo ? hi - lo4 : 0u;
                const uint32_t bulk = span & ~3u;
                const bool fits = span <= uint32_t(L::kVCap);
                if (lane == 0) {
                    vBase[vslot] = fits ? lo4 : 0xFFFFFFFFu;
                    if (fits && bulk != 0) {
                        dev::fenceProxyAsyncShared(); // earlier generic reads of the slot before the copy
                        dev::mbarArriveExpectTx(barV + 8 * vslot, 4 * bulk);
                        dev::bulkCopyG2S(dev::smemAddr(v), matrix.values + lo4, 4 * bulk, barV + 8 * vslot);
                    } else {
                        dev::mbarArrive(barV + 8 * vslot);
                    }
                }
                if (fits && lane < span - bulk)
                    dev::cpAsync4(dev::smemAddr(v + 4 * (bulk + lane)), matrix.values + lo4 + bulk + lane, 4u);
                dev::cpAsyncArriveNoinc(barV + 8 * vslot);
                __syncwarp(); // the invalid marks above, before the row copies read the IDs
                // X rows: whole rows, kLanesPerRow lanes of 16 bytes each. Lane group q copies rows
                // kGroupRows * q .. + kGroupRows - 1 and reads their IDs four at a time; an invalid
                // slot copies nothing (its A columns keep stale, finite bytes, which meet an all-zero
                // row of B).
                constexpr int kGroupRows = L::kSlots / L::kRowsPerCopy;
                const uint32_t group = lane / L::kLanesPerRow;
                const uint32_t xdst = base + L::kXOff + xslot * L::kXSlotBytes + group * kGroupRows * L::kXRowStride +
                                      16 * (lane % L::kLanesPerRow);
                const int8_t* xsrc = packedX + 16 * (lane % L::kLanesPerRow);
                const uint4* gids = reinterpret_cast<const uint4*>(a) + group * (kGroupRows / 4);
#pragma unroll
                for (int i4 = 0; i4 < kGroupRows / 4; ++i4) {
                    const uint4 q = gids[i4];
                    const uint32_t id4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        dev::cpAsync16LineIf(xdst + (4 * i4 + k) * L::kXRowStride, xsrc + uint64_t(id4[k]) * F, id4[k],
                                             cols);
                }
                dev::cpAsyncArriveNoinc(barXF + 8 * xslot);
            }
            if (!ok)
                break;
            // ---- B step: the B tiles of chunk seqF, once the MMAs of chunk seqF - 1 are done.
            // Chunk c's commit goes to sFree[c % 2], so each producer waits on consecutive
            // phases of one barrier (the parity of a phase two ahead would be ambiguous). ----
            const uint32_t aslot = seqF % L::kARing, vslot = seqF % L::kVRing;
            if (!boundedWait(barV + 8 * vslot, (seqF / L::kVRing) & 1) ||
                (seqF >= 1 && !boundedWait(barS + 8 * ((seqF - 1) & 1), ((seqF - 1) >> 1) & 1))) {
                ok = false;
                break;
            }
            const unsigned char* a = smem + L::kAOff + aslot * L::kASlotBytes;
            const unsigned char* v = smem + L::kVOff + vslot * L::kVSlotBytes;
            const uint32_t np = reinterpret_cast<const uint32_t*>(a + L::kHeaderOff)[1];
            unsigned char* tiles = smem + L::kBOff;
            {
                uint4* z = reinterpret_cast<uint4*>(tiles);
#pragma unroll
                for (int i = 0; i < kChunk8 * L::kBTileBytes / 16 / 32; ++i)
                    z[i * 32 + lane] = make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
            const uint32_t vb = vBase[vslot];
            // Scatter of the chunk's nonzeros; `fetch(i)` gives value i of a slot's run. The source
            // of the values (the staged range, or global memory when it did not fit) is chosen
            // once per chunk, outside the per-nonzero loop.
            auto scatter = [&](auto fetch) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t slot = lane + 32 * h;
                    const uint32_t pp = slot >> 3, k = slot & 7;
                    const uint64_t meta =
                        pp < np ? reinterpret_cast<const uint64_t*>(a + 4 * L::kSlots)[slot] : 0ull;
                    const float scale = reinterpret_cast<const float*>(v + 4 * L::kVCap)[slot];
                    uint32_t mask = static_cast<uint32_t>(meta);
                    uint32_t i = static_cast<uint32_t>(meta >> 32);
                    uint32_t* tile =
                        reinterpret_cast<uint32_t*>(tiles + pp * L::kBTileBytes + (k >> 2) * 128 + (k & 3) * 4);
                    while (mask) {
                        const int r = __ffs(mask) - 1;
                        mask &= mask - 1;
                        const float b = __uint_as_float(dev::tf32Exact(fetch(i++))) * scale;
                        const uint32_t bh = dev::tf32Exact(b);
                        const uint32_t bl = dev::tf32Exact(b - __uint_as_float(bh));
                        tile[((r & 7) * 16 + (r >> 3) * 256) / 4] = bh;
                        tile[((r & 7) * 16 + (r >> 3) * 256 + 1024) / 4] = bl;
                    }
                }
            };
            if (vb != 0xFFFFFFFFu) {
                const float* vsm = reinterpret_cast<const float*>(v);
                scatter([&](uint32_t i) { return vsm[i - vb]; });
            } else {
                scatter([&](uint32_t i) { return __ldg(matrix.values + i); });
            }
            dev::fenceProxyAsyncShared();
            __syncwarp();
            if (lane == 0)
                dev::mbarArrive(barB);
        }
        if (!ok)
            flags[1] = 1;
        dev::cpAsyncWaitAll();
        // No bulk copy may still be writing into this CTA's shared memory at exit: the value
        // ranges of V steps whose B step did not run (a wait ran out) and the IDs and metadata
        // of A steps. A phase already waited for returns at once.
        for (uint32_t s = seqV >= L::kVRing + pw ? seqV - L::kVRing : pw; s < seqV; s += P)
            boundedWait(barV + 8 * (s % L::kVRing), (s / L::kVRing) & 1);
        for (uint32_t s = seqA >= L::kARing + pw ? seqA - L::kARing : pw; s < seqA; s += P)
            boundedWait(barL + 8 * (s % L::kARing), (s / L::kARing) & 1);
    } else if (warp == L::kMmaWarp) {
        // ================================ MMA issuer (one warp) ============================
        // The whole warp runs the issue loop in uniform control flow and one lane, chosen by
        // elect.sync, issues each tcgen05 instruction. The issuer is on the critical chain of every
        // chunk (A columns and B tiles in, commit out) and shares its SM sub-partition with seven
        // other warps, so its instruction count per chunk is kept minimal: descriptors stepped by
        // a constant, the instruction descriptor an immediate, full chunks fully unrolled.
        bool ok = true, issued = false;
        uint32_t seq = 0, windows = 0;
        // Failure-path test (kTestStallOddCtas): the MMA warp of every odd CTA first waits on the
        // drain barrier, which nothing completes before the end, so that wait runs out and the
        // other roles' waits for its commits run out after it. Every wait stays bounded; the CTA
        // drains its copies, frees its tensor memory and returns.
        if ((testFlags & kTestStallOddCtas) && (blockIdx.x & 1u))
            ok = boundedWait(barF, 0);
        const unsigned long long desc0 = bTileDesc(base + L::kBOff);
        constexpr uint32_t kTileStep = L::kBTileBytes >> 4; // descriptor units between B tiles
        // The next task's panel range is loaded one task ahead, off the MMA issue path.
        uint32_t nextBegin = 0, nextEnd = 0;
        if (blockIdx.x < matrix.taskCount) {
            nextBegin = matrix.tasks[blockIdx.x].begin;
            nextEnd = matrix.tasks[blockIdx.x].end;
        }
        for (uint64_t tk = blockIdx.x; tk < matrix.taskCount; tk += gridDim.x) {
            const uint32_t panelCount = nextEnd - nextBegin;
            if (tk + gridDim.x < matrix.taskCount) {
                nextBegin = matrix.tasks[tk + gridDim.x].begin;
                nextEnd = matrix.tasks[tk + gridDim.x].end;
            }
            if (panelCount == 0)
                continue;
            if (ok && windows >= 1 && !boundedWait(barR, (windows - 1) & 1))
                ok = false;
            ++windows;
            dev::tcFenceAfter();
            const uint32_t nch = (panelCount + kChunk8 - 1) / kChunk8;
            for (uint32_t ch = 0; ch < nch; ++ch, ++seq) {
                // These waits are on the critical path: suspend on the barrier (resumes at once)
                // rather than sleep between polls.
                if (ok && (!boundedWait(barA, seq & 1) || !boundedWait(barB, seq & 1)))
                    ok = false;
                if (!ok)
                    continue;
                dev::tcFenceAfter();
                const uint32_t inChunk = min(uint32_t(kChunk8), panelCount - ch * kChunk8);
                if (inChunk == kChunk8) {
#pragma unroll
                    for (int sl = 0; sl < L::kSlices; ++sl)
                        dev::mmaTf32Chunk8Elected<L::kIdesc, 8, kTileStep>(
                            tmem + sl * L::kSliceCols + 8 * kChunk8, tmem + sl * L::kSliceCols, desc0, ch != 0);
                } else {
                    for (uint32_t pp = 0; pp < inChunk; ++pp)
#pragma unroll
                        for (int sl = 0; sl < L::kSlices; ++sl)
                            dev::mmaTf32TsElected<L::kIdesc>(tmem + sl * L::kSliceCols + 8 * kChunk8,
                                                             tmem + sl * L::kSliceCols + 8 * pp,
                                                             desc0 + pp * kTileStep, (ch | pp) != 0);
                }
                issued = true;
                dev::tcCommitElected(barS + 8 * (seq & 1));
            }
            if (ok)
                dev::tcCommitElected(barD);
        }
        if (issued) { // every MMA is complete before the tensor memory is released
            dev::tcCommitElected(barF);
            if (!boundedWait(barF, 0))
                ok = false;
        }
        if (!ok)
            flags[1] = 1;
        __syncwarp();
    } else {
        // ==================================== consumers ===================================
        const int quarter = warp & 3, slice = warp >> 2;
        const int g = lane >> 2, c = lane & 3;
        const uint32_t tLane = uint32_t(32 * quarter) << 16;
        const uint32_t aTmem = tmem + slice * L::kSliceCols + tLane;
        const uint32_t dTmem = tmem + slice * L::kSliceCols + 8 * kChunk8 + tLane;
        const uint32_t feature = slice * 128 + 32 * quarter + tmemLaneFeature(lane);
        // Word g of this warp's 32 bytes (128 * slice + 32 * quarter) of row 2c of panel 0; row
        // 2c + 1 follows one row stride later, panel pp 8 row strides later.
        const uint32_t xLane = base + L::kXOff + 2 * c * L::kXRowStride + 32 * warp + 4 * g;
        bool ok = true;
        uint32_t seq = 0, windows = 0;
        uint32_t xSlot = 0, xPhase = 0; // X slot of chunk seq (seq % kXDepth) and its phase parity
        tcc_sw32_task nextTask{};
        if (blockIdx.x < matrix.taskCount)
            nextTask = matrix.tasks[blockIdx.x];
        for (uint64_t tk = blockIdx.x; tk < matrix.taskCount; tk += gridDim.x) {
            const tcc_sw32_task task = nextTask;
            if (tk + gridDim.x < matrix.taskCount)
                nextTask = matrix.tasks[tk + gridDim.x];
            const uint32_t panelCount = task.end - task.begin;
            const uint32_t nch = (panelCount + kChunk8 - 1) / kChunk8;
            for (uint32_t ch = 0; ch < nch; ++ch, ++seq) {
                // The chunk's X rows have landed, and the MMAs of chunk seq - 1 are complete: the A
                // columns may be rewritten (the producer refills the B tiles at the same time).
                const uint32_t xslot = xSlot, xparity = xPhase;
                if (++xSlot == uint32_t(L::kXDepth)) {
                    xSlot = 0;
                    xPhase ^= 1u;
                }
                if (ok && (!boundedWait(barXF + 8 * xslot, xparity) ||
                           (seq >= 1 && !boundedWait(barS + 8 * ((seq - 1) & 1), ((seq - 1) >> 1) & 1))))
                    ok = false;
                if (!ok)
                    continue;
                dev::tcFenceAfter();
                const uint32_t xs = xLane + xslot * L::kXSlotBytes;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t lo[16], hi[16];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int pp = 4 * half + q;
                        const uint32_t wa = dev::ldsU32(xs + 8 * L::kXRowStride * pp) ^ 0x80808080u;
                        const uint32_t wb = dev::ldsU32(xs + 8 * L::kXRowStride * pp + L::kXRowStride) ^ 0x80808080u;
                        dev::int8PairToFloat<0>(wa, wb, lo[4 * q + 0], lo[4 * q + 1]);
                        dev::int8PairToFloat<1>(wa, wb, lo[4 * q + 2], lo[4 * q + 3]);
                        dev::int8PairToFloat<2>(wa, wb, hi[4 * q + 0], hi[4 * q + 1]);
                        dev::int8PairToFloat<3>(wa, wb, hi[4 * q + 2], hi[4 * q + 3]);
                    }
                    dev::tcStore16x256bx4(aTmem + 32 * half, lo);
                    dev::tcStore16x256bx4(aTmem + 32 * half + (16u << 16), hi);
                }
                dev::tcWaitSt();
                dev::tcFenceBefore();
                __syncwarp();
                dev::mbarArriveIf(lane == 0, barA);
                dev::mbarArriveIf(lane == 0, barXE + 8 * xslot); // the chunk's X rows are read
            }
            // ---- epilogue of this window ----
            if (task.sw == kSkipTask) // a padding entry: no panels (no chunks above), no rows
                continue;
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
                if (!split && rowBase + 32 <= rows) {
                    // Unsplit window with all 32 rows in range (all but the last window): 16
                    // branch-free stores at constant offsets from one row pointer. The epilogue
                    // sits between a window's last commit and the next window's first A columns.
                    float* out = output + uint64_t(rowBase + 16 * half) * F + feature;
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        __stcs(out + j * F, __uint_as_float(h[j]) + __uint_as_float(l[j]));
                    continue;
                }
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
