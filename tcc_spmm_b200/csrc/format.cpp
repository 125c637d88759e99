// Host construction of the SW32 panel format, its task plan and canonical CSR.
//
// The output is byte-identical to the reference (Shixg-cnic/tcc_spmm):
//   convertCsrToSw32   src/format/sw32.cpp:69-167
//   buildPanelTasks    src/format/sw32.cpp:25-65
//   makeCanonicalCsr   src/format/csr.cpp:6-40
// The reference builds the format in one sequential pass with a per-window k-way heap
// merge. Here every 32-row window (SW) is independent, so the build runs in three passes
// over the windows: (1) per-window bucket sizes, in parallel; (2) a prefix sum that fixes
// every window's panel and value offsets; (3) the fill, in parallel, each window writing
// only its own ranges. Within a window the entries are ordered by (source, row) with a
// sort, which yields exactly the order of the reference's merge for valid input.
#include "common.hpp"
#include "format/csr.h"
#include "format/sw32.h"

#include <cmath>
#include <cstring>
#include <limits>
#include <mutex>
#include <queue>

namespace tcc {
namespace {

constexpr std::uint32_t kNoPartial = 0xFFFFFFFFu;
constexpr std::uint32_t kPaddingSource = 0xFFFFFFFFu;
constexpr std::uint32_t kSkipTaskWindow = 0xFFFFFFFFu; // padding entry of a persistent task order

std::uint32_t to32(std::uint64_t n) {
    if (n > std::numeric_limits<std::uint32_t>::max())
        throw std::overflow_error("source-mask format exceeds uint32 offsets");
    return static_cast<std::uint32_t>(n);
}

// The first failure in window (or row) order among parallel workers.
class FirstError {
  public:
    void record(std::uint64_t where, int kind, const char* message) {
        std::lock_guard<std::mutex> lock(mutex_);
        if (!set_ || where < where_) {
            set_ = true;
            where_ = where;
            kind_ = kind;
            message_ = message;
        }
    }
    void rethrow() const {
        if (!set_)
            return;
        if (kind_ == TCC_OVERFLOW)
            throw std::overflow_error(message_);
        throw std::invalid_argument(message_);
    }

  private:
    std::mutex mutex_;
    bool set_ = false;
    std::uint64_t where_ = 0;
    int kind_ = 0;
    std::string message_;
};

// 4-bit mask of the 8-row groups touched by a 32-bit destination-row mask.
inline unsigned rowGroupsOf(std::uint32_t rowMask) {
    return unsigned((rowMask & 0x000000FFu) != 0) | (unsigned((rowMask & 0x0000FF00u) != 0) << 1) |
           (unsigned((rowMask & 0x00FF0000u) != 0) << 2) |
           (unsigned((rowMask & 0xFF000000u) != 0) << 3);
}

struct Entry {
    std::uint32_t source, row, pos;
};

// For a window with invalid entries: replay the reference's k-way merge order (sources
// ascending, rows ascending within a source; a row's next entry enters only after its
// previous one left) and return the message of the first violation it meets
// (reference src/format/sw32.cpp:102-123). Only runs on invalid input.
const char* firstMergeError(std::uint32_t base, std::uint32_t count, std::uint32_t cols, const std::uint32_t* offsets,
                            const std::uint32_t* sources, const float* values) {
    auto later = [](const Entry& a, const Entry& b) {
        return a.source > b.source || (a.source == b.source && a.row > b.row);
    };
    std::vector<Entry> heap;
    for (std::uint32_t r = 0; r < count; ++r)
        if (offsets[base + r] != offsets[base + r + 1])
            heap.push_back({sources[offsets[base + r]], r, offsets[base + r]});
    std::make_heap(heap.begin(), heap.end(), later);
    while (!heap.empty()) {
        const std::uint32_t source = heap.front().source;
        if (source >= cols)
            return "source-mask source outside column range";
        do {
            std::pop_heap(heap.begin(), heap.end(), later);
            Entry node = heap.back();
            heap.pop_back();
            const float v = values[node.pos];
            if (!std::isfinite(v) || v == 0.0f)
                return "source-mask requires finite nonzero values";
            if (++node.pos < offsets[base + node.row + 1]) {
                node.source = sources[node.pos];
                if (node.source <= source)
                    return "source-mask requires increasing row sources";
                heap.push_back(node);
                std::push_heap(heap.begin(), heap.end(), later);
            }
        } while (!heap.empty() && heap.front().source == source);
    }
    return "invalid canonical CSR for source-mask SW32";
}

// One window's entries ordered by (source, local row); validates them against the rules
// of the reference merge. Returns false (and records the error) on invalid input.
struct WindowScratch {
    std::vector<Entry> entries;
    // Item i: distinct source, its row mask and the position of its first entry.
    std::vector<std::uint32_t> itemSource, itemMask, itemFirst;
    std::vector<std::uint32_t> bucketItems[16];

    bool gather(std::uint32_t sw, std::uint32_t rows, std::uint32_t cols, const std::uint32_t* offsets,
                const std::uint32_t* sources, const float* values, bool bucketed, FirstError& error) {
        entries.clear();
        itemSource.clear();
        itemMask.clear();
        itemFirst.clear();
        for (auto& b : bucketItems)
            b.clear();
        const std::uint64_t base = std::uint64_t(sw) * 32;
        const std::uint32_t count = static_cast<std::uint32_t>(std::min<std::uint64_t>(32, rows - base));
        bool anomaly = false;
        for (std::uint32_t r = 0; r < count; ++r) {
            const std::uint32_t row = static_cast<std::uint32_t>(base) + r;
            const std::uint32_t lo = offsets[row], hi = offsets[row + 1];
            for (std::uint32_t p = lo; p < hi; ++p) {
                const float v = values[p];
                anomaly |= (p > lo && sources[p] <= sources[p - 1]) || sources[p] >= cols || !std::isfinite(v) ||
                           v == 0.0f;
                entries.push_back({sources[p], r, p});
            }
        }
        if (anomaly) {
            // Report the error the reference's merge meets first.
            error.record(sw, TCC_INVALID_ARGUMENT, firstMergeError(static_cast<std::uint32_t>(base), count, cols,
                                                                   offsets, sources, values));
            return false;
        }
        std::sort(entries.begin(), entries.end(), [](const Entry& a, const Entry& b) {
            return a.source < b.source || (a.source == b.source && a.row < b.row);
        });
        for (std::size_t i = 0; i < entries.size(); ++i) {
            const Entry& e = entries[i];
            if (i == 0 || e.source != entries[i - 1].source) {
                itemSource.push_back(e.source);
                itemMask.push_back(0);
                itemFirst.push_back(static_cast<std::uint32_t>(i));
            }
            itemMask.back() |= 1u << e.row;
        }
        for (std::uint32_t item = 0; item < itemSource.size(); ++item)
            bucketItems[bucketed ? rowGroupsOf(itemMask[item]) : 0].push_back(item);
        return true;
    }
};

// Split heavy windows into tasks of at most sw32TaskPanelLimit panels and index their
// partial sums (reference src/format/sw32.cpp:25-65). Sequential and linear in the number
// of windows plus split chunks.
void buildTasks(Sw32HostFormat& out) {
    const std::uint32_t windows = to32(out.windowOffsets.size() - 1);
    out.tasks.clear();
    out.reductions.clear();
    out.partialIds.clear();
    out.tasks.reserve(windows);
    std::uint64_t parts = 0;
    std::vector<std::uint32_t> groupParts[4];
    for (std::uint32_t sw = 0; sw < windows; ++sw) {
        const std::uint32_t first = out.windowOffsets[sw], last = out.windowOffsets[sw + 1];
        const std::uint32_t panels = last - first;
        if (panels <= sw32TaskPanelLimit) {
            out.tasks.push_back({sw, first, last, kNoPartial, 15u, 1u, 0u});
            continue;
        }
        const std::uint32_t chunks = (panels + sw32TaskPanelLimit - 1) / sw32TaskPanelLimit;
        const std::uint32_t reduceFirst = to32(out.reductions.size());
        for (auto& g : groupParts)
            g.clear();
        const std::uint32_t* slotBegin = out.bucketOffsets.data() + std::size_t(sw) * 17;
        for (std::uint32_t begin = first; begin < last; begin += sw32TaskPanelLimit) {
            const std::uint32_t end = begin + std::min(sw32TaskPanelLimit, last - begin);
            unsigned mask = 0;
            for (unsigned slot = 1; slot < 16; ++slot)
                if (std::max(begin, slotBegin[slot]) < std::min(end, slotBegin[slot + 1]))
                    mask |= sw32BucketOrder[slot];
            out.tasks.push_back({sw, begin, end, to32(parts), mask, chunks, reduceFirst});
            for (unsigned g = 0; g < 4; ++g)
                if (mask & (1u << g))
                    groupParts[g].push_back(to32(parts++));
        }
        for (const auto& g : groupParts) {
            const std::uint32_t from = to32(out.partialIds.size());
            out.partialIds.insert(out.partialIds.end(), g.begin(), g.end());
            out.reductions.push_back({from, to32(out.partialIds.size())});
        }
    }
    to32(out.tasks.size());
    to32(out.reductions.size());
    out.partialCount = to32(parts);
}

} // namespace

Sw32HostFormat convertCsr(std::uint32_t rows, std::uint32_t cols, const std::uint32_t* offsets,
                          const std::uint32_t* sources, const float* values, std::uint64_t nnz,
                          bool bucketed, unsigned threads) {
    if (rows == 0 || cols == 0 || offsets == nullptr || offsets[0] != 0 || offsets[rows] != nnz ||
        (nnz != 0 && (sources == nullptr || values == nullptr)))
        throw std::invalid_argument("invalid canonical CSR for source-mask SW32");
    for (std::uint32_t r = 0; r < rows; ++r)
        if (offsets[r] > offsets[r + 1])
            throw std::invalid_argument("decreasing CSR offsets");

    const std::uint32_t windows = static_cast<std::uint32_t>((std::uint64_t(rows) + 31) / 32);
    const unsigned orderCount = bucketed ? 16u : 1u;
    // Pass 1: items per bucket of every window -> panels per bucket slot.
    std::vector<std::uint32_t> slotPanels(std::size_t(windows) * 16, 0);
    FirstError error;
    constexpr std::size_t grain = 64;
    parallelFor(windows, grain, threads, [&](std::size_t lo, std::size_t hi) {
        WindowScratch scratch;
        for (std::size_t sw = lo; sw < hi; ++sw) {
            if (!scratch.gather(static_cast<std::uint32_t>(sw), rows, cols, offsets, sources, values,
                                bucketed, error))
                return;
            for (unsigned s = 0; s < orderCount; ++s) {
                const auto n = scratch.bucketItems[bucketed ? sw32BucketOrder[s] : 0].size();
                slotPanels[sw * 16 + s] = static_cast<std::uint32_t>((n + 7) / 8);
            }
        }
    });
    error.rethrow();

    // Pass 2: window panel offsets (values follow the CSR: a window's values are the nnz
    // of its rows, so its first value index is the CSR offset of its first row).
    Sw32HostFormat out;
    out.rows = rows;
    out.cols = cols;
    out.windowOffsets.assign(std::size_t(windows) + 1, 0);
    std::uint64_t panels = 0;
    for (std::uint32_t sw = 0; sw < windows; ++sw) {
        for (unsigned s = 0; s < orderCount; ++s)
            panels += slotPanels[std::size_t(sw) * 16 + s];
        out.windowOffsets[sw + 1] = to32(panels);
    }
    to32(nnz);
    out.sourceIds.resize(panels * 8);
    out.sourceMetadata.resize(panels * 8);
    out.rowGroupMasks.resize(panels);
    out.values.resize(nnz);
    if (bucketed)
        out.bucketOffsets.resize(std::size_t(windows) * 17);

    // Pass 3: fill.
    parallelFor(windows, grain, threads, [&](std::size_t lo, std::size_t hi) {
        WindowScratch scratch;
        for (std::size_t sw = lo; sw < hi; ++sw) {
            scratch.gather(static_cast<std::uint32_t>(sw), rows, cols, offsets, sources, values,
                           bucketed, error);
            std::uint32_t panel = out.windowOffsets[sw];
            std::uint32_t valueIndex = offsets[std::min<std::uint64_t>(std::uint64_t(sw) * 32, rows)];
            for (unsigned s = 0; s < orderCount; ++s) {
                if (bucketed)
                    out.bucketOffsets[sw * 17 + s] = panel;
                const auto& items = scratch.bucketItems[bucketed ? sw32BucketOrder[s] : 0];
                std::size_t slot = std::size_t(panel) * 8;
                unsigned groups = 0, inPanel = 0;
                for (std::uint32_t item : items) {
                    const std::uint32_t mask = scratch.itemMask[item];
                    out.sourceIds[slot] = scratch.itemSource[item];
                    out.sourceMetadata[slot] = (std::uint64_t(valueIndex) << 32) | mask;
                    const unsigned n = static_cast<unsigned>(__builtin_popcount(mask));
                    const Entry* e = scratch.entries.data() + scratch.itemFirst[item];
                    for (unsigned k = 0; k < n; ++k)
                        out.values[valueIndex + k] = values[e[k].pos];
                    valueIndex += n;
                    ++slot;
                    groups |= rowGroupsOf(mask);
                    if (++inPanel == 8) {
                        out.rowGroupMasks[panel++] = groups;
                        groups = inPanel = 0;
                    }
                }
                if (inPanel != 0) {
                    for (; inPanel < 8; ++inPanel, ++slot) {
                        out.sourceIds[slot] = kPaddingSource;
                        out.sourceMetadata[slot] = 0;
                    }
                    out.rowGroupMasks[panel++] = groups;
                }
            }
            if (bucketed)
                out.bucketOffsets[sw * 17 + 16] = panel;
        }
    });
    if (bucketed)
        buildTasks(out);
    return out;
}

CsrMatrix canonicalCsr(std::uint32_t rows, std::uint32_t cols, std::uint32_t nnz,
                       const std::uint32_t* offsets, const std::uint32_t* sources, const float* values,
                       unsigned threads) {
    if (rows == 0 || cols == 0 || offsets == nullptr || offsets[0] != 0 || offsets[rows] != nnz)
        throw std::invalid_argument("invalid CSR dimensions or offsets");
    for (std::uint32_t row = 0; row < rows; ++row)
        if (offsets[row] > offsets[row + 1] || offsets[row + 1] > nnz)
            throw std::invalid_argument("invalid CSR offsets");

    // Rows are processed in blocks; every block keeps its output and the blocks are
    // concatenated in row order afterwards.
    constexpr std::size_t grain = 4096;
    const std::size_t blocks = (std::size_t(rows) + grain - 1) / grain;
    std::vector<std::vector<std::uint32_t>> blockCols(blocks), blockLens(blocks);
    std::vector<std::vector<float>> blockVals(blocks);
    FirstError error;
    parallelFor(rows, grain, threads, [&](std::size_t lo, std::size_t hi) {
        const std::size_t b = lo / grain;
        auto& bc = blockCols[b];
        auto& bv = blockVals[b];
        auto& bl = blockLens[b];
        bl.reserve(hi - lo);
        std::vector<std::pair<std::uint32_t, float>> row;
        for (std::size_t r = lo; r < hi; ++r) {
            row.clear();
            bool sorted = true;
            for (std::uint32_t e = offsets[r]; e < offsets[r + 1]; ++e) {
                if (sources[e] >= cols || !std::isfinite(values[e])) {
                    error.record(r, TCC_INVALID_ARGUMENT, "invalid CSR column or nonfinite value");
                    return;
                }
                if (!row.empty() && sources[e] < row.back().first)
                    sorted = false;
                row.emplace_back(sources[e], values[e]);
            }
            if (!sorted)
                std::stable_sort(row.begin(), row.end(),
                                 [](const auto& a, const auto& b) { return a.first < b.first; });
            std::uint32_t kept = 0;
            for (std::size_t i = 0; i < row.size();) {
                const std::uint32_t column = row[i].first;
                float sum = 0.0f;
                do {
                    sum += row[i++].second;
                } while (i < row.size() && row[i].first == column);
                if (!std::isfinite(sum)) {
                    error.record(r, TCC_INVALID_ARGUMENT, "nonfinite coalesced weight");
                    return;
                }
                if (sum != 0.0f) {
                    bc.push_back(column);
                    bv.push_back(sum);
                    ++kept;
                }
            }
            bl.push_back(kept);
        }
    });
    error.rethrow();
    CsrMatrix out;
    std::size_t total = 0;
    for (const auto& bc : blockCols)
        total += bc.size();
    out.rowOffsets.reserve(std::size_t(rows) + 1);
    out.sourceIds.reserve(total);
    out.values.reserve(total);
    std::uint32_t running = 0;
    for (std::size_t b = 0; b < blocks; ++b) {
        for (std::uint32_t len : blockLens[b]) {
            running += len;
            out.rowOffsets.push_back(running);
        }
        out.sourceIds.insert(out.sourceIds.end(), blockCols[b].begin(), blockCols[b].end());
        out.values.insert(out.values.end(), blockVals[b].begin(), blockVals[b].end());
    }
    return out;
}

// Estimated cost of a task, in units of about one panel's share of a chunk: the fast kernel works
// in 8-panel chunks, and a partly filled chunk costs about as much as a full one (80 per chunk);
// a panel whose sources touch several 8-row groups scatters more B entries (2 per extra group);
// and every task pays its window epilogue (accumulator read-out and row stores, about 2.7 chunks'
// time at F = 128 in a per-phase profile of the kernel: 220; a chunk of F = 256 carries two
// feature slices while the epilogue's length stays, so the term halves relative to the chunks).
double taskCost(const tcc_sw32_task& task, const std::uint32_t* masks, std::uint32_t features) {
    const std::uint32_t panels = task.end - task.begin;
    double cost = 220.0 * 128.0 / std::max(128u, features) + 80.0 * ((panels + 7) / 8);
    if (masks)
        for (std::uint32_t p = task.begin; p < task.end; ++p)
            cost += 2.0 * (__builtin_popcount(masks[p] & 15u) - 1);
    return cost;
}

// Balanced contiguous task ranges cut at window boundaries.
void partitionTasks(const tcc_sw32_task* tasks, std::uint32_t count, const std::uint32_t* masks,
                    std::uint32_t features, std::uint32_t parts, std::uint32_t* bounds) {
    if (parts == 0 || (count != 0 && tasks == nullptr))
        throw std::invalid_argument("invalid task partition request");
    std::vector<double> prefix(std::size_t(count) + 1, 0.0);
    for (std::uint32_t i = 0; i < count; ++i)
        prefix[i + 1] = prefix[i] + taskCost(tasks[i], masks, features);
    bounds[0] = 0;
    for (std::uint32_t k = 1; k < parts; ++k) {
        const double target = prefix[count] * k / parts;
        std::uint32_t cut = static_cast<std::uint32_t>(
            std::lower_bound(prefix.begin(), prefix.end(), target) - prefix.begin());
        cut = std::min(cut, count);
        // Never separate the chunks of one split window.
        while (cut > 0 && cut < count && tasks[cut].sw == tasks[cut - 1].sw)
            ++cut;
        bounds[k] = std::max(cut, bounds[k - 1]);
    }
    bounds[parts] = count;
}

// Task order for a persistent launch of `ctas` CTAs in which CTA b takes tasks b, b + G, b + 2G,
// ... (G = min(ctas, count)). The tasks are dealt heaviest first, in rounds of G: in each round
// every CTA receives one task, the heaviest remaining going to the CTA with the least estimated
// work so far, so the CTAs' task counts differ by at most one (the last, partial round goes to
// the least-loaded CTAs, which take the lowest indices). The result is a permutation of the
// input: the SpMM is independent of task order (every task writes only its own window's rows or
// partial blocks, and the split-window merge sums partials in the reduce ranges' fixed order).
void balanceTasks(const tcc_sw32_task* tasks, std::uint32_t count, const std::uint32_t* masks,
                  std::uint32_t features, std::uint32_t ctas, tcc_sw32_task* out) {
    if (ctas == 0 || (count != 0 && (tasks == nullptr || out == nullptr)))
        throw std::invalid_argument("invalid task balance request");
    if (count == 0)
        return;
    const std::uint32_t g = std::min(ctas, count);
    std::vector<double> cost(count);
    for (std::uint32_t i = 0; i < count; ++i)
        cost[i] = taskCost(tasks[i], masks, features);
    std::vector<std::uint32_t> order(count);
    for (std::uint32_t i = 0; i < count; ++i)
        order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](std::uint32_t a, std::uint32_t b) { return cost[a] > cost[b]; });
    std::vector<std::vector<std::uint32_t>> bins(g);
    std::vector<double> load(g, 0.0);
    std::vector<std::uint32_t> byLoad(g);
    for (std::uint32_t b = 0; b < g; ++b)
        byLoad[b] = b;
    for (std::uint32_t at = 0; at < count; at += g) {
        const std::uint32_t n = std::min(g, count - at);
        std::stable_sort(byLoad.begin(), byLoad.end(), [&](std::uint32_t a, std::uint32_t b) { return load[a] < load[b]; });
        for (std::uint32_t i = 0; i < n; ++i) {
            const std::uint32_t bin = byLoad[i], task = order[at + i];
            bins[bin].push_back(task);
            load[bin] += cost[task];
        }
    }
    // CTAs b < count % g take one task more: put the bins that received one first.
    const std::size_t full = count / g;
    std::vector<std::uint32_t> binOrder(g);
    for (std::uint32_t b = 0; b < g; ++b)
        binOrder[b] = b;
    std::stable_partition(binOrder.begin(), binOrder.end(), [&](std::uint32_t b) { return bins[b].size() > full; });
    for (std::uint32_t b = 0; b < g; ++b) {
        const auto& list = bins[binOrder[b]];
        for (std::size_t k = 0; k < list.size(); ++k)
            out[b + k * g] = tasks[list[k]];
    }
}

// Relative speed of the k-th resident CTA of an SM (k = b / (G / ctasPerSm) for CTA b of a
// full persistent grid of G CTAs, which the hardware makes resident in block order), measured
// on B200 for the tensor-memory kernel: the SM's schedulers favour the older CTAs' warps, so
// with equal work the fourth CTA of an SM takes 15% longer than the first (power-law and R-MAT
// alike); the speeds below are those seen once the work is dealt by them (power-law, stress).
// Other residencies get equal speeds.
double residentSpeed(std::uint32_t ctasPerSm, std::uint32_t k) {
    static const double four[4] = {1.0, 0.94, 0.90, 0.82};
    static const double two[2] = {1.0, 0.895};
    if (ctasPerSm == 4 && k < 4)
        return four[k];
    if (ctasPerSm == 2 && k < 2)
        return two[k];
    return 1.0;
}

// Task order for a persistent launch in which CTA b takes entries b, b + G, b + 2G, ... and
// CTAs run at the speeds of residentSpeed: tasks dealt heaviest first, each to the CTA that
// would finish it earliest (longest-processing-time on machines of different speeds), so the
// CTAs receive different numbers of tasks. CTA b's list is laid out at b + k * G; shorter lists
// are padded with entries of window kSkipTask (no panels, no rows) that every kernel skips.
// Returns the number of entries, G * (longest list); `out` may be null to query it.
std::uint32_t balanceTasksPadded(const tcc_sw32_task* tasks, std::uint32_t count, const std::uint32_t* masks,
                                 std::uint32_t features, std::uint32_t ctas, std::uint32_t ctasPerSm,
                                 tcc_sw32_task* out, std::uint64_t capacity) {
    if (ctas == 0 || ctasPerSm == 0 || (count != 0 && tasks == nullptr))
        throw std::invalid_argument("invalid task balance request");
    if (count == 0)
        return 0;
    const std::uint32_t g = std::min(ctas, count);
    const bool full = g == ctas && ctas % ctasPerSm == 0;
    const std::uint32_t perRank = full ? ctas / ctasPerSm : g;
    std::vector<double> cost(count);
    for (std::uint32_t i = 0; i < count; ++i)
        cost[i] = taskCost(tasks[i], masks, features);
    std::vector<std::uint32_t> order(count);
    for (std::uint32_t i = 0; i < count; ++i)
        order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](std::uint32_t a, std::uint32_t b) { return cost[a] > cost[b]; });
    // One min-heap of (load, CTA) per speed class: the earliest finish of a task is at the top of
    // one of them.
    const std::uint32_t classes = full ? ctasPerSm : 1;
    using Entry = std::pair<double, std::uint32_t>;
    std::vector<std::priority_queue<Entry, std::vector<Entry>, std::greater<Entry>>> heaps(classes);
    std::vector<double> speed(classes);
    for (std::uint32_t c = 0; c < classes; ++c)
        speed[c] = full ? residentSpeed(ctasPerSm, c) : 1.0;
    // The last kBoundary CTAs before each residency boundary are sometimes made resident after
    // the first ones of the next rank: deal them at the slower speed.
    constexpr std::uint32_t kBoundary = 12;
    for (std::uint32_t b = 0; b < g; ++b) {
        std::uint32_t c = full ? b / perRank : 0;
        if (full && c + 1 < classes && b % perRank >= perRank - std::min(kBoundary, perRank / 4))
            ++c;
        heaps[c].push({0.0, b});
    }
    std::vector<std::vector<std::uint32_t>> lists(g);
    for (std::uint32_t at = 0; at < count; ++at) {
        const std::uint32_t task = order[at];
        std::uint32_t best = 0;
        double bestFinish = 0.0;
        for (std::uint32_t c = 0; c < classes; ++c) {
            const double finish = (heaps[c].top().first + cost[task]) / speed[c];
            if (c == 0 || finish < bestFinish) {
                best = c;
                bestFinish = finish;
            }
        }
        Entry e = heaps[best].top();
        heaps[best].pop();
        lists[e.second].push_back(task);
        e.first += cost[task];
        heaps[best].push(e);
    }
    std::size_t longest = 0;
    for (const auto& l : lists)
        longest = std::max(longest, l.size());
    const std::uint64_t entries = std::uint64_t(g) * longest;
    if (entries > 0xFFFFFFFFull)
        throw std::invalid_argument("padded task order too long");
    if (out == nullptr)
        return static_cast<std::uint32_t>(entries);
    if (capacity < entries)
        throw std::invalid_argument("output capacity below the padded task count");
    const tcc_sw32_task skip{kSkipTaskWindow, 0, 0, kNoPartial, 0, 0, 0};
    for (std::uint32_t b = 0; b < g; ++b)
        for (std::size_t k = 0; k < longest; ++k)
            out[b + k * g] = k < lists[b].size() ? tasks[lists[b][k]] : skip;
    return static_cast<std::uint32_t>(entries);
}

} // namespace tcc

// ------------------------------------------------------------------------------------
// C++ drop-in API (reference signatures).
// ------------------------------------------------------------------------------------
Sw32HostFormat convertCsrToSw32(std::uint32_t rows, std::uint32_t cols, const CsrMatrix& csr,
                                bool bucketByRwMask) {
    if (csr.rowOffsets.size() != std::size_t(rows) + 1 || csr.values.size() != csr.sourceIds.size())
        throw std::invalid_argument("invalid canonical CSR for source-mask SW32");
    return tcc::convertCsr(rows, cols, csr.rowOffsets.data(), csr.sourceIds.data(), csr.values.data(),
                           csr.sourceIds.size(), bucketByRwMask, 0);
}

CsrMatrix makeCanonicalCsr(std::uint32_t rows, std::uint32_t cols, std::uint32_t nnz,
                           const std::uint32_t* rowOffsets, const std::uint32_t* sourceIds,
                           const float* values) {
    return tcc::canonicalCsr(rows, cols, nnz, rowOffsets, sourceIds, values, 0);
}
