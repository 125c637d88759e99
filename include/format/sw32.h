// SW32 panel format types, interface- and layout-compatible with the reference's
// include/format/sw32.h:1-56. The structs below are the device ABI of launchSpmmInt8:
// their layouts must not change (Sw32Task is 28 bytes, Sw32DeviceView is nine pointers
// followed by a u32).
#pragma once

#include "format/csr.h"
#include <cstdint>
#include <vector>

// Emission order of the 16 row-group-mask buckets of one 32-row window (SW): the empty
// mask, the four single-RW masks, then the masks shared by two or more 8-row groups.
inline constexpr unsigned sw32BucketOrder[16] = {0, 1, 2, 4, 8, 3, 5, 6,
                                                 7, 9, 10, 11, 12, 13, 14, 15};

// A window with more panels than this is split into contiguous tasks of at most this many.
inline constexpr std::uint32_t sw32TaskPanelLimit = 384;

// One CTA's work: panels [begin, end) of window sw. partial == UINT32_MAX for an unsplit
// window; otherwise the first partial-sum block of this task, mask its participating
// 8-row groups, chunks the number of tasks of the window and reduceFirst its first
// Sw32ReduceRange.
struct Sw32Task {
    std::uint32_t sw, begin, end, partial, mask, chunks, reduceFirst;
};
// A range of partialIds to be summed, in task order, into one 8-row group.
struct Sw32ReduceRange {
    std::uint32_t begin, end;
};

// Host storage of the format. Each panel holds 8 source slots; each slot carries its
// source ID, a 32-bit destination-row mask (low word of sourceMetadata) and the index of
// its first value (high word); the slot's values follow in increasing row order.
// Padding slots have sourceIds == UINT32_MAX and metadata 0.
struct Sw32HostFormat {
    std::uint32_t rows = 0, cols = 0;
    std::vector<std::uint32_t> windowOffsets{0}, sourceIds, rowGroupMasks;
    std::vector<std::uint64_t> sourceMetadata;
    std::vector<float> values;
    // With RW buckets: 17 absolute panel offsets per window; bucket slot s holds the
    // panels of mask sw32BucketOrder[s] in [offset[s], offset[s+1]).
    std::vector<std::uint32_t> bucketOffsets;
    // Tasks in natural window order, the merge ranges of split windows and their partials.
    std::vector<Sw32Task> tasks;
    std::vector<Sw32ReduceRange> reductions;
    std::vector<std::uint32_t> partialIds;
    std::uint32_t partialCount = 0;
};

// Build the format on the host. launchSpmmInt8 needs bucketByRwMask = true (the default),
// which also builds the task plan.
Sw32HostFormat convertCsrToSw32(std::uint32_t rows, std::uint32_t cols, const CsrMatrix& csr,
                                bool bucketByRwMask = true);

// Device addresses of the uploaded arrays above (non-owning).
struct Sw32DeviceView {
    const std::uint32_t *windowOffsets, *sourceIds, *rowGroupMasks;
    const std::uint64_t* sourceMetadata;
    const float* values;
    const std::uint32_t* bucketOffsets = nullptr;
    const Sw32Task* tasks = nullptr;
    const Sw32ReduceRange* reductions = nullptr;
    const std::uint32_t* partialIds = nullptr;
    std::uint32_t taskCount = 0;
};
