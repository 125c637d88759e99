// Seeded synthetic workloads with the shapes of the benchmark configurations (the reference
// measures on ogbn-products, which is not available here). Every random draw comes from a
// counter-based generator keyed by (seed, stream, index), so the output does not depend on
// the thread count. All generators emit canonical CSR directly: rows hold strictly
// increasing columns and nonzero finite values.
//
//   poisson : row nnz ~ Poisson(mean) at uniform columns, values U(-1,1) \ {0}
//   powerlaw: power-law out-degrees rescaled to an exact nnz target, a fraction of every
//             row's neighbours uniform within +-radius of the row and the rest uniform over
//             the other columns, values 1/sqrt(deg_i*deg_j)
//   stress  : light rows U[lo,hi] nnz at uniform columns plus heavy rows U[hlo,hhi] nnz
//             clustered into a few 32-row windows, values U(0,1]
//   rmat    : R-MAT(a,b,c,d) edge samples, duplicates merged, values 1/deg_i
#include "workloads.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace {

thread_local std::string lastError;

inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Counter-based stream: draw i of stream s under seed is mix64(seed ^ mix64(s) + i).
struct Stream {
    uint64_t key;
    uint64_t counter = 0;
    Stream(uint64_t seed, uint64_t stream) : key(mix64(seed ^ mix64(stream * 0xD6E8FEB86659FD93ull + 1))) {}
    uint64_t next() { return mix64(key + (counter++) * 0x9E3779B97F4A7C15ull); }
    double uniform() { return double(next() >> 11) * (1.0 / 9007199254740992.0); } // [0,1)
    uint32_t below(uint64_t n) { return static_cast<uint32_t>((unsigned __int128)(next()) * n >> 64); }
};

template <typename Body> void parallelRange(uint64_t n, uint64_t grain, unsigned threads, Body&& body) {
    if (n == 0)
        return;
    if (threads == 0)
        threads = std::max(1u, std::thread::hardware_concurrency());
    const uint64_t blocks = (n + grain - 1) / grain;
    threads = static_cast<unsigned>(std::min<uint64_t>(threads, blocks));
    std::atomic<uint64_t> next{0};
    std::exception_ptr failure;
    std::atomic<bool> failed{false};
    auto worker = [&] {
        try {
            for (;;) {
                const uint64_t b = next.fetch_add(1);
                if (b >= blocks || failed.load())
                    return;
                body(b * grain, std::min(n, (b + 1) * grain));
            }
        } catch (...) {
            if (!failed.exchange(true))
                failure = std::current_exception();
        }
    };
    std::vector<std::thread> pool;
    for (unsigned t = 1; t < threads; ++t)
        pool.emplace_back(worker);
    worker();
    for (auto& t : pool)
        t.join();
    if (failure)
        std::rethrow_exception(failure);
}

template <typename Body> int guarded(Body&& body) {
    try {
        lastError.clear();
        body();
        return 0;
    } catch (const std::exception& e) {
        lastError = e.what();
        return 1;
    } catch (...) {
        lastError = "unknown error";
        return 1;
    }
}

tcc_wl_csr* allocCsr(uint32_t rows, uint32_t cols, uint64_t nnz) {
    if (nnz > 0xFFFFFFFFull)
        throw std::overflow_error("nnz exceeds 32-bit CSR offsets");
    auto* out = static_cast<tcc_wl_csr*>(std::calloc(1, sizeof(tcc_wl_csr)));
    if (!out)
        throw std::bad_alloc();
    out->rows = rows;
    out->cols = cols;
    out->nnz = nnz;
    out->rowOffsets = static_cast<uint32_t*>(std::malloc((uint64_t(rows) + 1) * sizeof(uint32_t)));
    out->sourceIds = static_cast<uint32_t*>(std::malloc(std::max<uint64_t>(nnz, 1) * sizeof(uint32_t)));
    out->values = static_cast<float*>(std::malloc(std::max<uint64_t>(nnz, 1) * sizeof(float)));
    if (!out->rowOffsets || !out->sourceIds || !out->values) {
        tcc_wl_free(out);
        throw std::bad_alloc();
    }
    return out;
}

// Fill `out` with `count` distinct values of [0, n) (count <= n), sorted, drawn from `rng`.
void distinctSorted(Stream& rng, uint32_t n, uint32_t count, std::vector<uint32_t>& out) {
    out.clear();
    if (count == 0)
        return;
    if (uint64_t(count) * 2 > n) { // pick the complement instead
        std::vector<uint32_t> skip;
        distinctSorted(rng, n, n - count, skip);
        out.reserve(count);
        std::size_t s = 0;
        for (uint32_t v = 0; v < n; ++v) {
            if (s < skip.size() && skip[s] == v) {
                ++s;
                continue;
            }
            out.push_back(v);
        }
        return;
    }
    while (out.size() < count) {
        const std::size_t have = out.size();
        for (std::size_t i = have; i < count; ++i)
            out.push_back(rng.below(n));
        std::sort(out.begin(), out.end());
        out.erase(std::unique(out.begin(), out.end()), out.end());
    }
    // Trim any excess deterministically (cannot happen with the loop above, kept for safety).
    out.resize(count);
}

uint32_t poissonDraw(Stream& rng, double mean) {
    // Knuth's product method (mean is small for this generator).
    const double limit = std::exp(-mean);
    double product = rng.uniform();
    uint32_t k = 0;
    while (product > limit) {
        ++k;
        product *= rng.uniform();
    }
    return k;
}

} // namespace

// Error message of the calling thread's last failed call (shared with workloads_gpu.cu).
void tccWlSetLastError(const char* message) { lastError = message ? message : ""; }

extern "C" {

const char* tcc_wl_last_error(void) { return lastError.c_str(); }

void tcc_wl_free(tcc_wl_csr* csr) {
    if (!csr)
        return;
    std::free(csr->rowOffsets);
    std::free(csr->sourceIds);
    std::free(csr->values);
    std::free(csr);
}

int tcc_wl_poisson(uint32_t rows, uint32_t cols, double mean, uint64_t seed, uint32_t threads, tcc_wl_csr** out) {
    return guarded([&] {
        *out = nullptr;
        if (rows == 0 || cols == 0)
            throw std::invalid_argument("empty matrix");
        std::vector<uint32_t> degree(rows);
        parallelRange(rows, 4096, threads, [&](uint64_t lo, uint64_t hi) {
            for (uint64_t r = lo; r < hi; ++r) {
                Stream rng(seed, 3 * r);
                degree[r] = std::min(poissonDraw(rng, mean), cols);
            }
        });
        // Duplicated columns are drawn without replacement, so the degree is exact.
        uint64_t nnz = 0;
        for (uint32_t d : degree)
            nnz += d;
        tcc_wl_csr* csr = allocCsr(rows, cols, nnz);
        csr->rowOffsets[0] = 0;
        for (uint32_t r = 0; r < rows; ++r)
            csr->rowOffsets[r + 1] = csr->rowOffsets[r] + degree[r];
        parallelRange(rows, 4096, threads, [&](uint64_t lo, uint64_t hi) {
            std::vector<uint32_t> colsOut;
            for (uint64_t r = lo; r < hi; ++r) {
                Stream rc(seed, 3 * r + 1), rv(seed, 3 * r + 2);
                distinctSorted(rc, cols, degree[r], colsOut);
                const uint32_t off = csr->rowOffsets[r];
                for (uint32_t i = 0; i < degree[r]; ++i) {
                    csr->sourceIds[off + i] = colsOut[i];
                    float v;
                    do {
                        v = static_cast<float>(rv.uniform() * 2.0 - 1.0);
                    } while (v == 0.0f);
                    csr->values[off + i] = v;
                }
            }
        });
        *out = csr;
    });
}

int tcc_wl_powerlaw(uint32_t rows, uint64_t target_nnz, double alpha, uint32_t max_degree, double local_fraction,
                    uint32_t local_radius, uint64_t seed, uint32_t threads, tcc_wl_csr** out) {
    return guarded([&] {
        *out = nullptr;
        if (rows == 0 || alpha <= 1.0 || max_degree == 0)
            throw std::invalid_argument("invalid power-law parameters");
        const uint32_t cols = rows;
        const uint32_t cap = std::min(max_degree, cols);
        if (target_nnz > uint64_t(cap) * rows)
            throw std::invalid_argument("nnz target above rows * max_degree");
        // Raw Pareto(alpha, 1) degrees, then a scale c chosen so that sum(min(cap,
        // max(1, round(c * raw)))) reaches the target, then +-1 corrections.
        std::vector<double> raw(rows);
        parallelRange(rows, 8192, threads, [&](uint64_t lo, uint64_t hi) {
            for (uint64_t r = lo; r < hi; ++r) {
                Stream rng(seed, 4 * r);
                raw[r] = std::pow(1.0 - rng.uniform(), -1.0 / (alpha - 1.0));
            }
        });
        auto total = [&](double c) {
            uint64_t sum = 0;
            for (double x : raw)
                sum += std::min<uint64_t>(cap, std::max<uint64_t>(1, uint64_t(std::llround(c * x))));
            return sum;
        };
        double lo = 0.0, hi = 1.0;
        while (total(hi) < target_nnz && hi < 1e12)
            hi *= 2.0;
        for (int it = 0; it < 100; ++it) {
            const double mid = 0.5 * (lo + hi);
            (total(mid) < target_nnz ? lo : hi) = mid;
        }
        std::vector<uint32_t> degree(rows);
        uint64_t sum = 0;
        for (uint32_t r = 0; r < rows; ++r) {
            degree[r] = static_cast<uint32_t>(std::min<uint64_t>(cap, std::max<uint64_t>(1, uint64_t(std::llround(hi * raw[r])))));
            sum += degree[r];
        }
        Stream fix(seed, 0xF1F1F1F1ull);
        while (sum != target_nnz) {
            const uint32_t r = fix.below(rows);
            if (sum < target_nnz && degree[r] < cap) {
                ++degree[r];
                ++sum;
            } else if (sum > target_nnz && degree[r] > 1) {
                --degree[r];
                --sum;
            }
        }
        tcc_wl_csr* csr = allocCsr(rows, cols, target_nnz);
        csr->rowOffsets[0] = 0;
        for (uint32_t r = 0; r < rows; ++r)
            csr->rowOffsets[r + 1] = csr->rowOffsets[r] + degree[r];
        parallelRange(rows, 2048, threads, [&](uint64_t lo2, uint64_t hi2) {
            std::vector<uint32_t> local, global, merged;
            for (uint64_t r = lo2; r < hi2; ++r) {
                const uint32_t d = degree[r];
                const uint32_t wlo = r > local_radius ? uint32_t(r - local_radius) : 0u;
                const uint32_t whi = std::min<uint64_t>(cols - 1, r + local_radius);
                const uint32_t window = whi - wlo + 1;
                const uint32_t outside = cols - window;
                uint32_t nLocal = std::min<uint32_t>(window, uint32_t(std::llround(local_fraction * d)));
                uint32_t nGlobal = d - nLocal;
                if (nGlobal > outside) {
                    nGlobal = outside;
                    nLocal = d - nGlobal;
                }
                Stream rl(seed, 4 * r + 1), rg(seed, 4 * r + 2);
                distinctSorted(rl, window, nLocal, local);
                distinctSorted(rg, outside, nGlobal, global);
                merged.clear();
                for (uint32_t v : local)
                    merged.push_back(wlo + v);
                for (uint32_t v : global)
                    merged.push_back(v < wlo ? v : v + window);
                std::sort(merged.begin(), merged.end());
                const uint32_t off = csr->rowOffsets[r];
                std::memcpy(csr->sourceIds + off, merged.data(), d * sizeof(uint32_t));
            }
        });
        parallelRange(target_nnz, 1 << 20, threads, [&](uint64_t lo2, uint64_t hi2) {
            // Row of entry e by binary search of the offsets (once per block), then walk.
            uint32_t r = static_cast<uint32_t>(std::upper_bound(csr->rowOffsets, csr->rowOffsets + rows + 1, lo2) -
                                               csr->rowOffsets) - 1;
            for (uint64_t e = lo2; e < hi2; ++e) {
                while (csr->rowOffsets[r + 1] <= e)
                    ++r;
                const double di = degree[r], dj = degree[csr->sourceIds[e]];
                csr->values[e] = static_cast<float>(1.0 / std::sqrt(di * dj));
            }
        });
        *out = csr;
    });
}

int tcc_wl_stress(uint32_t rows, uint32_t light_lo, uint32_t light_hi, uint32_t heavy_rows, uint32_t heavy_windows,
                  uint32_t heavy_lo, uint32_t heavy_hi, uint64_t seed, uint32_t threads, tcc_wl_csr** out) {
    return guarded([&] {
        *out = nullptr;
        const uint32_t cols = rows;
        const uint32_t windows = (rows + 31) / 32;
        if (rows == 0 || light_lo > light_hi || heavy_lo > heavy_hi || heavy_hi > cols || heavy_windows > windows ||
            heavy_rows > uint64_t(heavy_windows) * 32 || heavy_rows < heavy_windows)
            throw std::invalid_argument("invalid stress parameters");
        // Heavy windows, then heavy rows: one per heavy window plus the rest spread at random.
        Stream pick(seed, 0xABCDEFull);
        std::vector<uint32_t> heavyWin;
        distinctSorted(pick, windows - (rows % 32 ? 1 : 0), heavy_windows, heavyWin);
        std::vector<char> heavy(rows, 0);
        uint32_t placed = 0;
        for (uint32_t w : heavyWin) {
            heavy[w * 32 + pick.below(32)] = 1;
            ++placed;
        }
        while (placed < heavy_rows) {
            const uint32_t row = heavyWin[pick.below(heavyWin.size())] * 32 + pick.below(32);
            if (!heavy[row]) {
                heavy[row] = 1;
                ++placed;
            }
        }
        std::vector<uint32_t> degree(rows);
        for (uint32_t r = 0; r < rows; ++r) {
            Stream rng(seed, 3 * uint64_t(r));
            degree[r] = heavy[r] ? heavy_lo + rng.below(heavy_hi - heavy_lo + 1)
                                 : std::min(cols, light_lo + rng.below(light_hi - light_lo + 1));
        }
        uint64_t nnz = 0;
        for (uint32_t d : degree)
            nnz += d;
        tcc_wl_csr* csr = allocCsr(rows, cols, nnz);
        csr->rowOffsets[0] = 0;
        for (uint32_t r = 0; r < rows; ++r)
            csr->rowOffsets[r + 1] = csr->rowOffsets[r] + degree[r];
        parallelRange(rows, 1024, threads, [&](uint64_t lo, uint64_t hi) {
            std::vector<uint32_t> colsOut;
            for (uint64_t r = lo; r < hi; ++r) {
                Stream rc(seed, 3 * r + 1), rv(seed, 3 * r + 2);
                distinctSorted(rc, cols, degree[r], colsOut);
                const uint32_t off = csr->rowOffsets[r];
                for (uint32_t i = 0; i < degree[r]; ++i) {
                    csr->sourceIds[off + i] = colsOut[i];
                    csr->values[off + i] = float((rv.next() >> 40) + 1) * (1.0f / 16777216.0f); // (0,1]
                }
            }
        });
        *out = csr;
    });
}

int tcc_wl_rmat(uint32_t scale, uint64_t edges, double a, double b, double c, uint64_t seed, uint32_t threads,
                tcc_wl_csr** out) {
    return guarded([&] {
        *out = nullptr;
        if (scale == 0 || scale > 31 || a < 0 || b < 0 || c < 0 || a + b + c > 1.0)
            throw std::invalid_argument("invalid R-MAT parameters");
        const uint32_t n = 1u << scale;
        // Sample edges in blocks; every block is bucketed by row into per-row counts first.
        const uint64_t block = 1ull << 22;
        const uint64_t blocks = (edges + block - 1) / block;
        std::vector<uint32_t> src(edges), dst(edges);
        const uint64_t ta = uint64_t(a * 18446744073709551615.0), tb = uint64_t((a + b) * 18446744073709551615.0),
                       tc = uint64_t((a + b + c) * 18446744073709551615.0);
        parallelRange(blocks, 1, threads, [&](uint64_t lo, uint64_t hi) {
            for (uint64_t bl = lo; bl < hi; ++bl) {
                Stream rng(seed, bl);
                const uint64_t e0 = bl * block, e1 = std::min(edges, e0 + block);
                for (uint64_t e = e0; e < e1; ++e) {
                    uint32_t r = 0, col = 0;
                    for (uint32_t level = 0; level < scale; ++level) {
                        const uint64_t u = rng.next();
                        const uint32_t bit = 1u << (scale - 1 - level);
                        if (u < ta) {
                        } else if (u < tb) {
                            col |= bit;
                        } else if (u < tc) {
                            r |= bit;
                        } else {
                            r |= bit;
                            col |= bit;
                        }
                    }
                    src[e] = r;
                    dst[e] = col;
                }
            }
        });
        // Counting sort by row, then sort + unique every row.
        std::vector<uint64_t> start(uint64_t(n) + 1, 0);
        for (uint64_t e = 0; e < edges; ++e)
            ++start[src[e] + 1];
        for (uint32_t r = 0; r < n; ++r)
            start[r + 1] += start[r];
        std::vector<uint32_t> byRow(edges);
        {
            std::vector<uint64_t> fill(start.begin(), start.end() - 1);
            for (uint64_t e = 0; e < edges; ++e)
                byRow[fill[src[e]]++] = dst[e];
        }
        std::vector<uint32_t>().swap(src);
        std::vector<uint32_t>().swap(dst);
        std::vector<uint32_t> degree(n);
        parallelRange(n, 4096, threads, [&](uint64_t lo, uint64_t hi) {
            for (uint64_t r = lo; r < hi; ++r) {
                uint32_t* first = byRow.data() + start[r];
                uint32_t* last = byRow.data() + start[r + 1];
                std::sort(first, last);
                degree[r] = static_cast<uint32_t>(std::unique(first, last) - first);
            }
        });
        uint64_t nnz = 0;
        for (uint32_t d : degree)
            nnz += d;
        tcc_wl_csr* csr = allocCsr(n, n, nnz);
        csr->rowOffsets[0] = 0;
        for (uint32_t r = 0; r < n; ++r)
            csr->rowOffsets[r + 1] = csr->rowOffsets[r] + degree[r];
        parallelRange(n, 4096, threads, [&](uint64_t lo, uint64_t hi) {
            for (uint64_t r = lo; r < hi; ++r) {
                const uint32_t off = csr->rowOffsets[r];
                const float v = degree[r] ? float(1.0 / degree[r]) : 0.0f;
                for (uint32_t i = 0; i < degree[r]; ++i) {
                    csr->sourceIds[off + i] = byRow[start[r] + i];
                    csr->values[off + i] = v;
                }
            }
        });
        *out = csr;
    });
}

int tcc_wl_normal(float* out, uint64_t count, uint64_t seed, uint32_t threads) {
    return guarded([&] {
        if (out == nullptr && count)
            throw std::invalid_argument("null output");
        parallelRange((count + 1) / 2, 1 << 16, threads, [&](uint64_t lo, uint64_t hi) {
            for (uint64_t i = lo; i < hi; ++i) {
                Stream rng(seed, i);
                // Box-Muller on two uniforms in (0,1].
                const double u1 = 1.0 - rng.uniform(), u2 = rng.uniform();
                const double radius = std::sqrt(-2.0 * std::log(u1));
                const double angle = 6.283185307179586 * u2;
                out[2 * i] = static_cast<float>(radius * std::cos(angle));
                if (2 * i + 1 < count)
                    out[2 * i + 1] = static_cast<float>(radius * std::sin(angle));
            }
        });
    });
}

} // extern "C"
