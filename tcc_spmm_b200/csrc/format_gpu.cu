// GPU construction of the SW32 panel format and its task plan from a canonical CSR that is
// already in device memory. The arrays are byte-identical to the host builder's (format.cpp),
// itself byte-identical to the reference (Shixg-cnic/tcc_spmm):
//   convertCsrToSw32   src/format/sw32.cpp:69-167
//   buildPanelTasks    src/format/sw32.cpp:25-65
// The reference merges the rows of each 32-row window (SW) with a heap on one host thread.
// Here the whole matrix is ordered at once, in five data-parallel steps:
//   1. every entry gets the key (window, source, local row); one radix sort orders all the
//      entries by it (the window bits on top keep the windows apart, the row bits at the
//      bottom order an item's values by row);
//   2. an item is a run of equal (window, source) keys: its first index is compacted, its row
//      mask is ORed over the run (at most 32 entries) and its bucket slot follows from the
//      mask's 8-row groups;
//   3. a stable radix sort by (window, slot) puts the items in emission order; a slot keeps
//      its items in source order because the sort is stable;
//   4. prefix sums give every (window, slot) its first panel and every item its first value:
//      emission order concatenates the windows, so the running nnz is the value index;
//   5. fill kernels write the slots, padding, row-group masks and bucket offsets, and one
//      thread per window writes its tasks, reduce ranges and partial IDs.
// Input validation gives the host builder's errors in the same order; for an invalid entry
// the first failing window is copied back and checked by the host builder, which yields the
// same message.
#include "common.hpp"
#include "format/sw32.h"

#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>
#include <cub/device/device_select.cuh>
#include <cuda_runtime.h>
#include <thrust/iterator/counting_iterator.h>

#include <limits>
#include <memory>
#include <mutex>
#include <vector>

namespace tcc {
Sw32HostFormat convertCsr(std::uint32_t rows, std::uint32_t cols, const std::uint32_t* offsets,
                          const std::uint32_t* sources, const float* values, std::uint64_t nnz,
                          bool bucketed, unsigned threads);
} // namespace tcc

struct tcc_sw32_device {
    void* block = nullptr; // one device allocation holding every array
    int device = 0;
    tcc_sw32_sizes sizes{};
    tcc_sw32_arrays arrays{};
};

namespace tcc {
namespace {

using u32 = std::uint32_t;
using u64 = std::uint64_t;

constexpr u32 kNoPartial = 0xFFFFFFFFu;
constexpr u32 kPaddingSource = 0xFFFFFFFFu;
constexpr unsigned kThreads = 256;

void throwIf(cudaError_t s) {
    if (s != cudaSuccess)
        throw CudaError(cudaGetErrorString(s));
}

struct ByteTable {
    unsigned char v[16];
};
constexpr ByteTable slotOfGroupsTable() {
    ByteTable t{};
    for (unsigned s = 0; s < 16; ++s)
        t.v[sw32BucketOrder[s]] = static_cast<unsigned char>(s);
    return t;
}
constexpr ByteTable groupsOfSlotTable() {
    ByteTable t{};
    for (unsigned s = 0; s < 16; ++s)
        t.v[s] = static_cast<unsigned char>(sw32BucketOrder[s]);
    return t;
}
// Bucket slot of a 4-bit row-group mask, and its inverse (the emission order).
__constant__ ByteTable gSlotOfGroups = slotOfGroupsTable();
__constant__ ByteTable gGroupsOfSlot = groupsOfSlotTable();

// Scalars the host reads back between the steps.
struct BuildStatus {
    u32 firstOffset, lastOffset; // offsets[0], offsets[rows]
    u32 decreasing;              // some offsets[r] > offsets[r + 1]
    u32 badWindow;               // first window holding an invalid entry (UINT32_MAX: none)
    u32 items;                   // distinct (window, source) pairs
    u32 tasks, parts, splits;    // task-plan totals
    u32 pad;
    u64 panels;                  // panels of the whole format
};

unsigned bitWidth(u64 v) {
    unsigned n = 0;
    while (v) {
        ++n;
        v >>= 1;
    }
    return n;
}

unsigned blocksFor(u64 threads) { return static_cast<unsigned>((threads + kThreads - 1) / kThreads); }

__device__ __forceinline__ unsigned rowGroupsOf(u32 m) {
    return unsigned((m & 0x000000FFu) != 0) | (unsigned((m & 0x0000FF00u) != 0) << 1) |
           (unsigned((m & 0x00FF0000u) != 0) << 2) | (unsigned((m & 0xFF000000u) != 0) << 3);
}

// offsets[0], offsets[rows] and whether the offsets ever decrease.
__global__ void checkOffsetsKernel(const u32* __restrict__ offsets, u32 rows, BuildStatus* st) {
    const u64 t = blockIdx.x * u64(blockDim.x) + threadIdx.x;
    if (t > rows)
        return;
    const u32 here = offsets[t];
    if (t < rows && here > offsets[t + 1])
        st->decreasing = 1;
    if (t == 0)
        st->firstOffset = here;
    if (t == rows)
        st->lastOffset = here;
}

// One warp per row: key = window << winShift | source << 5 | local row, value = CSR index.
// Flags the window of any entry the reference's merge rejects (source out of range, value
// zero or not finite, sources not strictly increasing along the row).
__global__ void entryKeysKernel(const u32* __restrict__ offsets, const u32* __restrict__ sources,
                                const float* __restrict__ values, u32 rows, u32 cols, unsigned winShift,
                                u64* __restrict__ keys, u32* __restrict__ pos, BuildStatus* st) {
    const u64 row = (blockIdx.x * u64(blockDim.x) + threadIdx.x) >> 5;
    const unsigned lane = threadIdx.x & 31;
    if (row >= rows)
        return; // warp-uniform
    const u64 lo = offsets[row], hi = offsets[row + 1];
    const u64 head = (u64(row >> 5) << winShift) | (row & 31);
    bool bad = false;
    for (u64 p = lo + lane; p < hi; p += 32) {
        const u32 s = sources[p];
        const float v = values[p];
        bad |= s >= cols || !isfinite(v) || v == 0.0f || (p > lo && sources[p - 1] >= s);
        keys[p] = head | (u64(s) << 5);
        pos[p] = static_cast<u32>(p);
    }
    if (__any_sync(0xFFFFFFFFu, bad) && lane == 0)
        atomicMin(&st->badWindow, static_cast<u32>(row >> 5));
}

struct IsItemHead {
    const u64* keys;
    __device__ bool operator()(u32 i) const { return i == 0 || (keys[i] >> 5) != (keys[i - 1] >> 5); }
};

// Per item: its row mask and its sort key (window << 4 | bucket slot).
__global__ void itemsKernel(const u64* __restrict__ keys, const u32* __restrict__ heads, u32 items, u32 nnz,
                            unsigned winShift, bool bucketed, u32* __restrict__ itemMask,
                            u32* __restrict__ itemKey, u32* __restrict__ perm) {
    const u64 j = blockIdx.x * u64(blockDim.x) + threadIdx.x;
    if (j >= items)
        return;
    const u32 first = heads[j], end = j + 1 < items ? heads[j + 1] : nnz;
    u32 mask = 0;
    for (u32 e = first; e < end; ++e)
        mask |= 1u << (static_cast<u32>(keys[e]) & 31u);
    const u32 window = static_cast<u32>(keys[first] >> winShift);
    const u32 slot = bucketed ? gSlotOfGroups.v[rowGroupsOf(mask)] : 0u;
    itemMask[j] = mask;
    itemKey[j] = (window << 4) | slot;
    perm[j] = static_cast<u32>(j);
}

// Item range of every (window, slot) in emission order, and each item's value count.
__global__ void runsKernel(const u32* __restrict__ sortedKey, const u32* __restrict__ perm,
                           const u32* __restrict__ itemMask, u32 items, u32* __restrict__ runStart,
                           u32* __restrict__ runEnd, u32* __restrict__ valueCount) {
    const u64 j = blockIdx.x * u64(blockDim.x) + threadIdx.x;
    if (j >= items)
        return;
    const u32 k = sortedKey[j];
    if (j == 0 || sortedKey[j - 1] != k)
        runStart[k] = static_cast<u32>(j);
    if (j + 1 == items || sortedKey[j + 1] != k)
        runEnd[k] = static_cast<u32>(j + 1);
    valueCount[j] = __popc(itemMask[perm[j]]);
}

// Panels of every (window, slot); the trailing element is 0 so that the exclusive sum's last
// element is the total.
__global__ void slotPanelsKernel(const u32* __restrict__ runStart, const u32* __restrict__ runEnd, u64 slots,
                                 u64* __restrict__ panels) {
    const u64 ws = blockIdx.x * u64(blockDim.x) + threadIdx.x;
    if (ws > slots)
        return;
    panels[ws] = ws < slots ? (u64(runEnd[ws] - runStart[ws]) + 7) / 8 : 0;
}

// Row-group mask of the panels [begin, end) of a window whose bucket slots start at slotBegin
// (the reference's rule: every bucket slot 1..15 that overlaps the range adds its groups).
__device__ __forceinline__ u32 chunkMask(const u64* slotBegin, u64 begin, u64 end) {
    u32 mask = 0;
    for (unsigned slot = 1; slot < 16; ++slot)
        if (max(begin, slotBegin[slot]) < min(end, slotBegin[slot + 1]))
            mask |= gGroupsOfSlot.v[slot];
    return mask;
}

// Tasks, partial sums and split flag of every window (trailing zeros for the sums).
__global__ void taskCountsKernel(const u64* __restrict__ panelStart, u32 windows, u32* __restrict__ tasks,
                                 u32* __restrict__ parts, u32* __restrict__ splits) {
    const u64 w = blockIdx.x * u64(blockDim.x) + threadIdx.x;
    if (w > windows)
        return;
    if (w == windows) {
        tasks[w] = parts[w] = splits[w] = 0;
        return;
    }
    const u64* slotBegin = panelStart + w * 16;
    const u64 first = slotBegin[0], last = slotBegin[16], panels = last - first;
    if (panels <= sw32TaskPanelLimit) {
        tasks[w] = 1;
        parts[w] = splits[w] = 0;
        return;
    }
    u32 chunks = 0, count = 0;
    for (u64 begin = first; begin < last; begin += sw32TaskPanelLimit, ++chunks)
        count += __popc(chunkMask(slotBegin, begin, min(begin + sw32TaskPanelLimit, last)));
    tasks[w] = chunks;
    parts[w] = count;
    splits[w] = 1;
}

// Slots, metadata and values of every item.
__global__ void fillItemsKernel(const u64* __restrict__ keys, const u32* __restrict__ pos,
                                const float* __restrict__ csrValues, const u32* __restrict__ heads,
                                const u32* __restrict__ itemMask, const u32* __restrict__ sortedKey,
                                const u32* __restrict__ perm, const u32* __restrict__ runStart,
                                const u64* __restrict__ panelStart, const u32* __restrict__ valueIndex, u32 items,
                                u64 sourceMask, bool bucketed, u32* __restrict__ sourceIds,
                                u64* __restrict__ metadata, float* __restrict__ values,
                                u32* __restrict__ rowGroupMasks) {
    const u64 j = blockIdx.x * u64(blockDim.x) + threadIdx.x;
    if (j >= items)
        return;
    const u32 id = perm[j], ws = sortedKey[j];
    const u32 first = heads[id], mask = itemMask[id];
    const u64 slot = panelStart[ws] * 8 + (j - runStart[ws]);
    const u32 vi = valueIndex[j];
    sourceIds[slot] = static_cast<u32>((keys[first] >> 5) & sourceMask);
    metadata[slot] = (u64(vi) << 32) | mask;
    const unsigned n = __popc(mask);
    for (unsigned e = 0; e < n; ++e)
        values[vi + e] = csrValues[pos[first + e]];
    if (!bucketed)
        atomicOr(&rowGroupMasks[slot >> 3], rowGroupsOf(mask));
}

// One warp per (window, slot): padding of its last panel, row-group masks (bucketed: the
// slot's groups), bucket offsets and window offsets.
__global__ void fillSlotsKernel(const u32* __restrict__ runStart, const u32* __restrict__ runEnd,
                                const u64* __restrict__ panelStart, u32 windows, bool bucketed,
                                u32* __restrict__ sourceIds, u64* __restrict__ metadata,
                                u32* __restrict__ rowGroupMasks, u32* __restrict__ bucketOffsets,
                                u32* __restrict__ windowOffsets) {
    const u64 ws = (blockIdx.x * u64(blockDim.x) + threadIdx.x) >> 5;
    const unsigned lane = threadIdx.x & 31;
    const u64 slots = u64(windows) * 16;
    if (ws >= slots)
        return;
    const u64 start = panelStart[ws], end = panelStart[ws + 1];
    const u32 count = runEnd[ws] - runStart[ws];
    const u32 w = static_cast<u32>(ws >> 4), s = static_cast<u32>(ws & 15);
    for (u64 q = start * 8 + count + lane; q < end * 8; q += 32) {
        sourceIds[q] = kPaddingSource;
        metadata[q] = 0;
    }
    if (bucketed) {
        const u32 groups = gGroupsOfSlot.v[s];
        for (u64 p = start + lane; p < end; p += 32)
            rowGroupMasks[p] = groups;
    }
    if (lane != 0)
        return;
    if (bucketed) {
        bucketOffsets[u64(w) * 17 + s] = static_cast<u32>(start);
        if (s == 15)
            bucketOffsets[u64(w) * 17 + 16] = static_cast<u32>(end);
    }
    if (s == 0)
        windowOffsets[w] = static_cast<u32>(start);
    if (ws + 1 == slots)
        windowOffsets[windows] = static_cast<u32>(end);
}

// The task plan of one window (reference buildPanelTasks, src/format/sw32.cpp:25-65): one
// task for up to sw32TaskPanelLimit panels; otherwise one task per chunk, each chunk owning
// one partial block per 8-row group it touches, and four reduce ranges listing the window's
// partial blocks per group in chunk order.
__global__ void fillTasksKernel(const u64* __restrict__ panelStart, const u32* __restrict__ taskStart,
                                const u32* __restrict__ partStart, const u32* __restrict__ splitStart,
                                u32 windows, tcc_sw32_task* __restrict__ tasks,
                                tcc_sw32_reduce_range* __restrict__ reductions, u32* __restrict__ partialIds) {
    const u64 w = blockIdx.x * u64(blockDim.x) + threadIdx.x;
    if (w >= windows)
        return;
    const u64* slotBegin = panelStart + w * 16;
    const u32 first = static_cast<u32>(slotBegin[0]), last = static_cast<u32>(slotBegin[16]);
    const u32 t = taskStart[w];
    if (last - first <= sw32TaskPanelLimit) {
        tasks[t] = {static_cast<u32>(w), first, last, kNoPartial, 15u, 1u, 0u};
        return;
    }
    const u32 chunks = (last - first + sw32TaskPanelLimit - 1) / sw32TaskPanelLimit;
    const u32 reduceFirst = 4 * splitStart[w], part0 = partStart[w];
    u32 part = part0, groupCount[4] = {0, 0, 0, 0};
    for (u32 c = 0; c < chunks; ++c) {
        const u32 begin = first + c * sw32TaskPanelLimit, end = min(begin + sw32TaskPanelLimit, last);
        const u32 mask = chunkMask(slotBegin, begin, end);
        tasks[t + c] = {static_cast<u32>(w), begin, end, part, mask, chunks, reduceFirst};
        for (unsigned g = 0; g < 4; ++g)
            groupCount[g] += (mask >> g) & 1u;
        part += __popc(mask);
    }
    u32 cursor[4];
    cursor[0] = part0;
    for (unsigned g = 1; g < 4; ++g)
        cursor[g] = cursor[g - 1] + groupCount[g - 1];
    for (unsigned g = 0; g < 4; ++g)
        reductions[reduceFirst + g] = {cursor[g], cursor[g] + groupCount[g]};
    part = part0;
    for (u32 c = 0; c < chunks; ++c) {
        const u32 begin = first + c * sw32TaskPanelLimit, end = min(begin + sw32TaskPanelLimit, last);
        const u32 mask = chunkMask(slotBegin, begin, end);
        for (unsigned g = 0; g < 4; ++g)
            if (mask & (1u << g))
                partialIds[cursor[g]++] = part++;
    }
}

// The builder's device memory comes from a pool of this library, one per device, that keeps
// what is freed into it (release threshold: unlimited), so that a later build maps no new
// memory; tcc_sw32_device_trim() hands the unused part back to the device.
constexpr int kMaxDevices = 64;
std::mutex gPoolMutex;
cudaMemPool_t gPools[kMaxDevices] = {};

cudaMemPool_t builderPool(int device, bool create) {
    if (device < 0 || device >= kMaxDevices)
        throw CudaError("device ordinal out of range");
    std::lock_guard<std::mutex> lock(gPoolMutex);
    if (gPools[device] == nullptr && create) {
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = device;
        cudaMemPool_t pool = nullptr;
        throwIf(cudaMemPoolCreate(&pool, &props));
        u64 keep = ~u64(0);
        throwIf(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
        gPools[device] = pool;
    }
    return gPools[device];
}

// Stream-ordered scratch from the builder's pool, released in stream order when the build
// returns or throws (or earlier, through release()).
class Scratch {
  public:
    Scratch(cudaMemPool_t pool, cudaStream_t stream) : pool_(pool), stream_(stream) {}
    Scratch(const Scratch&) = delete;
    Scratch& operator=(const Scratch&) = delete;
    ~Scratch() {
        for (void* p : blocks_)
            cudaFreeAsync(p, stream_);
    }
    template <typename T> T* get(u64 count) {
        void* p = nullptr;
        throwIf(cudaMallocFromPoolAsync(&p, std::max<u64>(count * sizeof(T), 16), pool_, stream_));
        blocks_.push_back(p);
        return static_cast<T*>(p);
    }
    void* bytes(std::size_t n) { return get<unsigned char>(n); }
    void release(void* p) {
        auto it = std::find(blocks_.begin(), blocks_.end(), p);
        if (it == blocks_.end())
            return;
        blocks_.erase(it);
        throwIf(cudaFreeAsync(p, stream_));
    }

  private:
    cudaMemPool_t pool_;
    cudaStream_t stream_;
    std::vector<void*> blocks_;
};

void syncRead(void* host, const void* device, std::size_t bytes, cudaStream_t stream) {
    throwIf(cudaMemcpyAsync(host, device, bytes, cudaMemcpyDeviceToHost, stream));
    throwIf(cudaStreamSynchronize(stream));
}

// Exact message of the host builder for the first invalid window (error path only).
[[noreturn]] void throwWindowError(u32 window, u32 rows, u32 cols, const u32* offsets, const u32* sources,
                                   const float* values, bool bucketed, cudaStream_t stream) {
    const u32 base = window * 32, count = std::min<u32>(32, rows - base);
    std::vector<u32> off(count + 1);
    syncRead(off.data(), offsets + base, sizeof(u32) * (count + 1), stream);
    const u32 n = off[count] - off[0];
    std::vector<u32> src(n);
    std::vector<float> val(n);
    if (n != 0) {
        syncRead(src.data(), sources + off[0], sizeof(u32) * n, stream);
        syncRead(val.data(), values + off[0], sizeof(float) * n, stream);
    }
    for (u32 r = count + 1; r-- > 0;)
        off[r] -= off[0];
    convertCsr(count, cols, off.data(), src.data(), val.data(), n, bucketed, 1);
    throw std::invalid_argument("invalid canonical CSR for source-mask SW32");
}

template <typename T> T* carve(unsigned char*& cursor, u64 count) {
    T* p = reinterpret_cast<T*>(cursor);
    cursor += (std::max<u64>(count * sizeof(T), 1) + 255) / 256 * 256;
    return p;
}

using DeviceFormat = std::unique_ptr<tcc_sw32_device, void (*)(tcc_sw32_device*)>;

DeviceFormat buildOnDevice(u32 rows, u32 cols, const u32* offsets, const u32* sources,
                                                const float* values, u64 nnz, bool bucketed,
                                                cudaStream_t stream) {
    if (rows == 0 || cols == 0 || offsets == nullptr || (nnz != 0 && (sources == nullptr || values == nullptr)))
        throw std::invalid_argument("invalid canonical CSR for source-mask SW32");
    DeviceFormat out(new tcc_sw32_device, tcc_sw32_device_free);
    throwIf(cudaGetDevice(&out->device));
    cudaMemPool_t pool = builderPool(out->device, true);
    Scratch scratch(pool, stream);
    BuildStatus* st = scratch.get<BuildStatus>(1);
    BuildStatus hs{};
    throwIf(cudaMemsetAsync(st, 0, sizeof(BuildStatus), stream));
    throwIf(cudaMemsetAsync(&st->badWindow, 0xFF, sizeof(u32), stream));

    // Offsets first: the key pass reads rows by them.
    checkOffsetsKernel<<<blocksFor(u64(rows) + 1), kThreads, 0, stream>>>(offsets, rows, st);
    throwIf(cudaGetLastError());
    syncRead(&hs, st, sizeof(hs), stream);
    if (hs.firstOffset != 0 || hs.lastOffset != nnz)
        throw std::invalid_argument("invalid canonical CSR for source-mask SW32");
    if (hs.decreasing)
        throw std::invalid_argument("decreasing CSR offsets");

    const u32 windows = static_cast<u32>((u64(rows) + 31) / 32);
    const u64 slots = u64(windows) * 16;
    const unsigned sourceBits = bitWidth(cols - 1), winShift = 5 + sourceBits;
    const unsigned windowBits = bitWidth(windows - 1);
    const u64 sourceMask = sourceBits >= 32 ? 0xFFFFFFFFull : ((1ull << sourceBits) - 1);
    const u32 n = static_cast<u32>(nnz); // offsets are u32, so nnz == offsets[rows] < 2^32

    // 1. Entry keys, validation, and the sort of all entries by (window, source, row).
    u64* keys = nullptr;
    u32* pos = nullptr;
    u32* heads = nullptr;
    u32 items = 0;
    if (n != 0) {
        u64* keyA = scratch.get<u64>(n);
        u64* keyB = scratch.get<u64>(n);
        u32* posA = scratch.get<u32>(n);
        u32* posB = scratch.get<u32>(n);
        entryKeysKernel<<<blocksFor(u64(rows) * 32), kThreads, 0, stream>>>(offsets, sources, values, rows, cols,
                                                                             winShift, keyA, posA, st);
        throwIf(cudaGetLastError());
        syncRead(&hs, st, sizeof(hs), stream);
        if (hs.badWindow != 0xFFFFFFFFu)
            throwWindowError(hs.badWindow, rows, cols, offsets, sources, values, bucketed, stream);

        cub::DoubleBuffer<u64> keyBuf(keyA, keyB);
        cub::DoubleBuffer<u32> posBuf(posA, posB);
        // Only the window and source bits are sorted: the sort is stable and the entries come
        // in CSR order, so an item's entries stay in increasing row order.
        const int endBit = static_cast<int>(winShift + windowBits);
        std::size_t tempBytes = 0;
        throwIf(cub::DeviceRadixSort::SortPairs(nullptr, tempBytes, keyBuf, posBuf, n, 5, endBit, stream));
        void* temp = scratch.bytes(tempBytes);
        throwIf(cub::DeviceRadixSort::SortPairs(temp, tempBytes, keyBuf, posBuf, n, 5, endBit, stream));
        keys = keyBuf.Current();
        pos = posBuf.Current();
        scratch.release(temp);
        scratch.release(keyBuf.Alternate());
        scratch.release(posBuf.Alternate());

        // 2. Items: first entry of every run of equal (window, source).
        heads = scratch.get<u32>(n);
        tempBytes = 0;
        throwIf(cub::DeviceSelect::If(nullptr, tempBytes, thrust::counting_iterator<u32>(0), heads, &st->items,
                                      static_cast<std::int64_t>(n), IsItemHead{keys}, stream));
        throwIf(cub::DeviceSelect::If(scratch.bytes(tempBytes), tempBytes, thrust::counting_iterator<u32>(0), heads,
                                      &st->items, static_cast<std::int64_t>(n), IsItemHead{keys}, stream));
        syncRead(&hs, st, sizeof(hs), stream);
        items = hs.items;
    }

    u32* itemMask = scratch.get<u32>(items);
    u32* sortedKey = scratch.get<u32>(items);
    u32* perm = scratch.get<u32>(items);
    u32* valueIndex = scratch.get<u32>(items);
    u32* runStart = scratch.get<u32>(slots);
    u32* runEnd = scratch.get<u32>(slots);
    throwIf(cudaMemsetAsync(runStart, 0, sizeof(u32) * slots, stream));
    throwIf(cudaMemsetAsync(runEnd, 0, sizeof(u32) * slots, stream));
    if (items != 0) {
        itemsKernel<<<blocksFor(items), kThreads, 0, stream>>>(keys, heads, items, n, winShift, bucketed, itemMask,
                                                              sortedKey, perm);
        throwIf(cudaGetLastError());
        // 3. Emission order: stable sort of the items by (window, slot).
        if (bucketed) {
            u32* keyB = scratch.get<u32>(items);
            u32* permB = scratch.get<u32>(items);
            cub::DoubleBuffer<u32> keyBuf(sortedKey, keyB), permBuf(perm, permB);
            const int endBit = static_cast<int>(4 + windowBits);
            std::size_t tempBytes = 0;
            throwIf(cub::DeviceRadixSort::SortPairs(nullptr, tempBytes, keyBuf, permBuf, items, 0, endBit, stream));
            void* temp = scratch.bytes(tempBytes);
            throwIf(cub::DeviceRadixSort::SortPairs(temp, tempBytes, keyBuf, permBuf, items, 0, endBit, stream));
            sortedKey = keyBuf.Current();
            perm = permBuf.Current();
            scratch.release(temp);
            scratch.release(keyBuf.Alternate());
            scratch.release(permBuf.Alternate());
        }
        runsKernel<<<blocksFor(items), kThreads, 0, stream>>>(sortedKey, perm, itemMask, items, runStart, runEnd,
                                                             valueIndex);
        throwIf(cudaGetLastError());
        // 4a. First value of every item.
        std::size_t tempBytes = 0;
        throwIf(cub::DeviceScan::ExclusiveSum(nullptr, tempBytes, valueIndex, valueIndex, items, stream));
        throwIf(cub::DeviceScan::ExclusiveSum(scratch.bytes(tempBytes), tempBytes, valueIndex, valueIndex, items,
                                              stream));
    }

    // 4b. First panel of every (window, slot), then the task plan's per-window counts.
    u64* panelStart = scratch.get<u64>(slots + 1);
    slotPanelsKernel<<<blocksFor(slots + 1), kThreads, 0, stream>>>(runStart, runEnd, slots, panelStart);
    throwIf(cudaGetLastError());
    {
        std::size_t tempBytes = 0;
        throwIf(cub::DeviceScan::ExclusiveSum(nullptr, tempBytes, panelStart, panelStart, slots + 1, stream));
        throwIf(cub::DeviceScan::ExclusiveSum(scratch.bytes(tempBytes), tempBytes, panelStart, panelStart, slots + 1,
                                              stream));
    }
    u32* taskStart = scratch.get<u32>(u64(windows) + 1);
    u32* partStart = scratch.get<u32>(u64(windows) + 1);
    u32* splitStart = scratch.get<u32>(u64(windows) + 1);
    throwIf(cudaMemcpyAsync(&st->panels, panelStart + slots, sizeof(u64), cudaMemcpyDeviceToDevice, stream));
    if (bucketed) {
        taskCountsKernel<<<blocksFor(u64(windows) + 1), kThreads, 0, stream>>>(panelStart, windows, taskStart,
                                                                                partStart, splitStart);
        throwIf(cudaGetLastError());
        for (u32* a : {taskStart, partStart, splitStart}) {
            std::size_t tempBytes = 0;
            throwIf(cub::DeviceScan::ExclusiveSum(nullptr, tempBytes, a, a, u64(windows) + 1, stream));
            throwIf(cub::DeviceScan::ExclusiveSum(scratch.bytes(tempBytes), tempBytes, a, a, u64(windows) + 1,
                                                  stream));
        }
    }
    if (bucketed) {
        throwIf(cudaMemcpyAsync(&st->tasks, taskStart + windows, sizeof(u32), cudaMemcpyDeviceToDevice, stream));
        throwIf(cudaMemcpyAsync(&st->parts, partStart + windows, sizeof(u32), cudaMemcpyDeviceToDevice, stream));
        throwIf(cudaMemcpyAsync(&st->splits, splitStart + windows, sizeof(u32), cudaMemcpyDeviceToDevice, stream));
    }
    syncRead(&hs, st, sizeof(hs), stream);
    const u64 panels = hs.panels;
    if (panels > std::numeric_limits<u32>::max())
        throw std::overflow_error("source-mask format exceeds uint32 offsets");

    // Outputs: one allocation, every array 256-byte aligned and non-null even when empty.
    tcc_sw32_sizes& z = out->sizes;
    z.rows = rows;
    z.cols = cols;
    z.partialCount = hs.parts;
    z.bucketed = bucketed ? 1u : 0u;
    z.windowOffsets = u64(windows) + 1;
    z.sourceIds = panels * 8;
    z.rowGroupMasks = panels;
    z.values = n;
    z.bucketOffsets = bucketed ? u64(windows) * 17 : 0;
    z.tasks = hs.tasks;
    z.reductions = u64(hs.splits) * 4;
    z.partialIds = hs.parts;
    const u64 total = 256 * 9 + 4 * z.windowOffsets + 12 * z.sourceIds + 4 * z.rowGroupMasks + 4 * z.values +
                      4 * z.bucketOffsets + sizeof(tcc_sw32_task) * z.tasks + 8 * z.reductions + 4 * z.partialIds;
    throwIf(cudaMallocFromPoolAsync(&out->block, total, pool, stream));
    unsigned char* cursor = static_cast<unsigned char*>(out->block);
    u32* windowOffsets = carve<u32>(cursor, z.windowOffsets);
    u32* sourceIds = carve<u32>(cursor, z.sourceIds);
    u64* metadata = carve<u64>(cursor, z.sourceIds);
    u32* rowGroupMasks = carve<u32>(cursor, z.rowGroupMasks);
    float* outValues = carve<float>(cursor, z.values);
    u32* bucketOffsets = carve<u32>(cursor, z.bucketOffsets);
    auto* tasks = carve<tcc_sw32_task>(cursor, z.tasks);
    auto* reductions = carve<tcc_sw32_reduce_range>(cursor, z.reductions);
    u32* partialIds = carve<u32>(cursor, z.partialIds);
    out->arrays = {windowOffsets, sourceIds, rowGroupMasks, metadata, outValues,
                   bucketOffsets, tasks,     reductions,    partialIds};

    // 5. Fill.
    if (!bucketed)
        throwIf(cudaMemsetAsync(rowGroupMasks, 0, sizeof(u32) * panels, stream));
    if (items != 0) {
        fillItemsKernel<<<blocksFor(items), kThreads, 0, stream>>>(
            keys, pos, values, heads, itemMask, sortedKey, perm, runStart, panelStart, valueIndex, items, sourceMask,
            bucketed, sourceIds, metadata, outValues, rowGroupMasks);
        throwIf(cudaGetLastError());
    }
    fillSlotsKernel<<<blocksFor(slots * 32), kThreads, 0, stream>>>(runStart, runEnd, panelStart, windows, bucketed,
                                                                     sourceIds, metadata, rowGroupMasks,
                                                                     bucketOffsets, windowOffsets);
    throwIf(cudaGetLastError());
    if (bucketed) {
        fillTasksKernel<<<blocksFor(windows), kThreads, 0, stream>>>(panelStart, taskStart, partStart, splitStart,
                                                                     windows, tasks, reductions, partialIds);
        throwIf(cudaGetLastError());
    }
    return out;
}

} // namespace
} // namespace tcc

extern "C" {

int tcc_convert_csr_to_sw32_device(uint32_t rows, uint32_t cols, const uint32_t* row_offsets,
                                   const uint32_t* source_ids, const float* values, uint64_t nnz,
                                   int bucket_by_rw_mask, tcc_stream_t stream, tcc_sw32_device** out) {
    return tcc::guarded([&] {
        if (out == nullptr)
            throw std::invalid_argument("null output handle");
        *out = nullptr;
        auto built = tcc::buildOnDevice(rows, cols, row_offsets, source_ids, values, nnz, bucket_by_rw_mask != 0,
                                        reinterpret_cast<cudaStream_t>(stream));
        *out = built.release();
    });
}

int tcc_sw32_device_sizes(const tcc_sw32_device* format, tcc_sw32_sizes* sizes) {
    return tcc::guarded([&] {
        if (format == nullptr || sizes == nullptr)
            throw std::invalid_argument("null argument");
        *sizes = format->sizes;
    });
}

int tcc_sw32_device_arrays(const tcc_sw32_device* format, tcc_sw32_arrays* arrays) {
    return tcc::guarded([&] {
        if (format == nullptr || arrays == nullptr)
            throw std::invalid_argument("null argument");
        *arrays = format->arrays;
    });
}

int tcc_sw32_device_view_of(const tcc_sw32_device* format, tcc_sw32_device_view* view) {
    return tcc::guarded([&] {
        if (format == nullptr || view == nullptr)
            throw std::invalid_argument("null argument");
        const tcc_sw32_arrays& a = format->arrays;
        *view = {a.windowOffsets, a.sourceIds,  a.rowGroupMasks, a.sourceMetadata,
                 a.values,        a.bucketOffsets, a.tasks,      a.reductions,
                 a.partialIds,    static_cast<uint32_t>(format->sizes.tasks)};
    });
}

void tcc_sw32_device_free(tcc_sw32_device* format) {
    if (format == nullptr)
        return;
    int current = 0;
    if (format->block != nullptr && cudaGetDevice(&current) == cudaSuccess) {
        // Work on any stream may still read the arrays: wait for the device, then hand the
        // block back to the builder's pool.
        cudaSetDevice(format->device);
        cudaDeviceSynchronize();
        cudaFreeAsync(format->block, nullptr);
        cudaStreamSynchronize(nullptr);
        cudaSetDevice(current);
    }
    delete format;
}

int tcc_sw32_device_trim(void) {
    return tcc::guarded([&] {
        int device = 0;
        tcc::throwIf(cudaGetDevice(&device));
        if (cudaMemPool_t pool = tcc::builderPool(device, false))
            tcc::throwIf(cudaMemPoolTrimTo(pool, 0));
    });
}

} // extern "C"
