// Device helpers of the SpMM kernels: TF32 operand preparation, the m16n8k8 TF32 MMA,
// packed f32x2 arithmetic, mbarriers and asynchronous copies (sm_100a inline PTX).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace tcc {
namespace dev {

// ---- TF32 operands ----------------------------------------------------------------------
// The reference rounds both MMA operands with cvt.rna.tf32.f32 (round to 10 mantissa bits,
// ties away from zero; reference src/kernel/spmm_kernel.cuh:7-11). Adding half a TF32 ulp
// (0x1000) to the FP32 bit pattern and dropping the low 13 bits is the same rounding for
// finite values: the carry out of the kept bits implements "half away from zero" on the
// magnitude. The tensor core ignores the low 13 bits of a TF32 operand, so the hot loop only
// adds; tf32Exact also clears them (used where the value is stored or compared).
__device__ __forceinline__ uint32_t tf32Biased(float v) { return __float_as_uint(v) + 0x1000u; }
__device__ __forceinline__ uint32_t tf32Exact(float v) {
    return (__float_as_uint(v) + 0x1000u) & 0xFFFFE000u;
}

// D(16x8) += A(16x8, row-major) * B(8x8, column-major), TF32 inputs, FP32 accumulate.
__device__ __forceinline__ void mmaTf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Shared-memory loads by 32-bit shared address (always LDS, cheap address arithmetic).
__device__ __forceinline__ uint32_t ldsU32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ uint2 ldsV2(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ uint4 ldsV4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
                 : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ldsU64(uint32_t addr) {
    unsigned long long v;
    asm volatile("ld.shared.u64 %0, [%1];" : "=l"(v) : "r"(addr) : "memory");
    return v;
}

// ---- packed FP32 pairs (sm_100a add/mul .f32x2) -----------------------------------------
__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
    return (static_cast<unsigned long long>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long mul2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint32_t lo32(unsigned long long v) { return static_cast<uint32_t>(v); }
__device__ __forceinline__ uint32_t hi32(unsigned long long v) { return static_cast<uint32_t>(v >> 32); }

// Dequantize the four INT8 features of one 32-bit word of a source row to biased TF32:
// out[i] = tf32(float(q_i) * scale). The signed byte is flipped to an unsigned one
// (q + 128), placed in the mantissa of 2^23 (exact float 2^23 + q + 128) and the offset is
// subtracted exactly, so float(q_i) costs one byte permute and half a packed add. The
// product is one IEEE multiply like the reference's float(int8) * multiplier.
__device__ __forceinline__ void dequant4(uint32_t word, unsigned long long scale2, uint32_t (&out)[4]) {
    const uint32_t w = word ^ 0x80808080u;
    const uint32_t magic = 0x4B000000u;
    const unsigned long long bias2 = 0xCB000080CB000080ull; // (-8388736.f, -8388736.f)
    const unsigned long long p01 =
        (static_cast<unsigned long long>(__byte_perm(w, magic, 0x7541)) << 32) | __byte_perm(w, magic, 0x7540);
    const unsigned long long p23 =
        (static_cast<unsigned long long>(__byte_perm(w, magic, 0x7543)) << 32) | __byte_perm(w, magic, 0x7542);
    const unsigned long long f01 = mul2(add2(p01, bias2), scale2);
    const unsigned long long f23 = mul2(add2(p23, bias2), scale2);
    out[0] = lo32(f01) + 0x1000u;
    out[1] = hi32(f01) + 0x1000u;
    out[2] = lo32(f23) + 0x1000u;
    out[3] = hi32(f23) + 0x1000u;
}

// ---- shared memory, mbarriers, async copies ----------------------------------------------
__device__ __forceinline__ uint32_t smemAddr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbarInit(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbarArrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Arrive on `bar` in the threads where `pred` holds, as one predicated instruction (no branch).
__device__ __forceinline__ void mbarArriveIf(bool pred, uint32_t bar) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %1, 0;\n\t@p mbarrier.arrive.shared::cta.b64 _, [%0];\n\t}" ::"r"(bar),
                 "r"(static_cast<uint32_t>(pred))
                 : "memory");
}
__device__ __forceinline__ bool mbarTryWait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done)
                 : "r"(bar), "r"(parity)
                 : "memory");
    return done != 0;
}
// try_wait that lets the hardware suspend the warp for up to `hintNs` nanoseconds (it resumes
// as soon as the phase completes), so waiting warps do not take issue slots.
__device__ __forceinline__ bool mbarTryWaitSuspend(uint32_t bar, uint32_t parity, uint32_t hintNs) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done)
                 : "r"(bar), "r"(parity), "r"(hintNs)
                 : "memory");
    return done != 0;
}
__device__ __forceinline__ uint64_t globalTimerNs() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Arrive on `bar` once every cp.async issued so far by this thread has landed. The barrier's
// expected count includes this arrival.
__device__ __forceinline__ void cpAsyncArriveNoinc(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
// 4-byte async copy; srcBytes 0 writes zero.
__device__ __forceinline__ void cpAsync4(uint32_t dst, const void* src, uint32_t srcBytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(srcBytes)
                 : "memory");
}
// L2 eviction policies (createpolicy): keep the gathered feature rows, stream the format. Used
// by the 4-panel and mma.sync kernels; the 8-panel default kernel runs faster without them.
__device__ __forceinline__ uint64_t policyEvictLast() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policyEvictFirst() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// 16-byte async copy with an L2 policy and a 128-byte L2 prefetch of the enclosing line.
__device__ __forceinline__ void cpAsync16Hint(uint32_t dst, const void* src, uint32_t srcBytes, uint64_t policy) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint.L2::128B [%0], [%1], 16, %2, %3;" ::"r"(dst), "l"(src),
                 "r"(srcBytes), "l"(policy)
                 : "memory");
}
// 16-byte async copy with a 128-byte L2 prefetch of the enclosing line and the default L2
// policy; srcBytes 0 writes zeros.
__device__ __forceinline__ void cpAsync16Line(uint32_t dst, const void* src, uint32_t srcBytes) {
    asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(srcBytes)
                 : "memory");
}
// cpAsync16Line issued only where id < limit, as one predicated instruction (no branch); the
// source address is formed but not read where the predicate fails.
__device__ __forceinline__ void cpAsync16LineIf(uint32_t dst, const void* src, uint32_t id, uint32_t limit) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.lt.u32 p, %2, %3;\n\t"
                 "@p cp.async.cg.shared.global.L2::128B [%0], [%1], 16;\n\t}" ::"r"(dst),
                 "l"(src), "r"(id), "r"(limit)
                 : "memory");
}
// A 4-byte cp.async issued only where id < limit (predicated, no branch).
__device__ __forceinline__ void cpAsync4If(uint32_t dst, const void* src, uint32_t id, uint32_t limit) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.lt.u32 p, %2, %3;\n\t"
                 "@p cp.async.ca.shared.global [%0], [%1], 4;\n\t}" ::"r"(dst), "l"(src), "r"(id), "r"(limit)
                 : "memory");
}
// 16 zero bytes to shared memory (16-byte aligned address).
__device__ __forceinline__ void stsZero16(uint32_t addr) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0u) : "memory");
}
__device__ __forceinline__ void cpAsync4Hint(uint32_t dst, const void* src, uint32_t srcBytes, uint64_t policy) {
    asm volatile("cp.async.ca.shared.global.L2::cache_hint [%0], [%1], 4, %2, %3;" ::"r"(dst), "l"(src), "r"(srcBytes),
                 "l"(policy)
                 : "memory");
}
__device__ __forceinline__ void cpAsync8Hint(uint32_t dst, const void* src, uint64_t policy) {
    asm volatile("cp.async.ca.shared.global.L2::cache_hint [%0], [%1], 8, 8, %2;" ::"r"(dst), "l"(src), "l"(policy)
                 : "memory");
}
__device__ __forceinline__ void cpAsyncCommit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cpAsyncWaitGroup() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cpAsyncWaitAll() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Bulk (TMA engine) copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from
// global to this CTA's shared memory, completing as transaction bytes on `bar`. No
// multicast: every copy lands in the issuing CTA only.
__device__ __forceinline__ void bulkCopyG2S(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// Same with an L2 cache policy for the source lines.
__device__ __forceinline__ void bulkCopyG2SHint(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                                uint64_t policy) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(policy)
                 : "memory");
}
// Arrive on `bar` and add `bytes` to the transaction count its current phase waits for.
__device__ __forceinline__ void mbarArriveExpectTx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void fenceBarrierInit() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tensor memory and the 5th-generation tensor core (tcgen05) ---------------------------
// Allocate `cols` TMEM columns (power of two >= 32) for this CTA; the whole warp executes it
// and the TMEM address is written to shared memory at `dst`.
__device__ __forceinline__ void tmemAlloc(uint32_t dst, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst), "r"(cols)
                 : "memory");
}
__device__ __forceinline__ void tmemRelinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmemDealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tcFenceBefore() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tcFenceAfter() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tcWaitSt() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tcWaitLd() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Make this thread's generic-proxy shared-memory writes visible to the async proxy (the
// tensor core reads its shared-memory operand through it).
__device__ __forceinline__ void fenceProxyAsyncShared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Warp store of 16 TMEM lanes x 32 columns (16x256b shape, 4 repetitions along the columns):
// thread t writes lanes t/4 (r[4j], r[4j+1]) and t/4 + 8 (r[4j+2], r[4j+3]) at columns
// 8j + 2(t%4) and 8j + 2(t%4) + 1, j = 0..3.
__device__ __forceinline__ void tcStore16x256bx4(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile("tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], "
                 "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
                 "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
                 : "memory");
}
// The same store with 2 repetitions (16 columns, 8 registers per thread).
__device__ __forceinline__ void tcStore16x256bx2(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.16x256b.x2.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
// Warp load of 32 TMEM lanes x 16 columns (32x32b shape, 16 repetitions): thread t reads
// lane t, r[j] = column j.
__device__ __forceinline__ void tcLoad32x32bx16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15])
                 : "r"(taddr)
                 : "memory");
}
// Byte K (K = 0..3) of two source words as exact floats: the packed f32x2 pair holds
// float(q) of source a's and source b's byte. The words are already flipped to unsigned
// bytes (word ^ 0x80808080); every int8 is exactly representable in TF32.
template <int K>
__device__ __forceinline__ void int8PairToFloat(uint32_t wa, uint32_t wb, uint32_t& outA, uint32_t& outB) {
    const uint32_t magic = 0x4B000000u;
    const unsigned long long bias2 = 0xCB000080CB000080ull; // (-8388736.f, -8388736.f)
    const unsigned long long p = (static_cast<unsigned long long>(__byte_perm(wb, magic, 0x7540 + K)) << 32) |
                                 __byte_perm(wa, magic, 0x7540 + K);
    const unsigned long long f = add2(p, bias2);
    outA = lo32(f);
    outB = hi32(f);
}

// D(tmem, M x N, FP32) (+)= A(tmem, M x K, TF32, K-major) * B(smem descriptor, K x N, TF32),
// one CTA, issued by a single thread. accumulate == 0 overwrites D.
__device__ __forceinline__ void mmaTf32Ts(uint32_t dTmem, uint32_t aTmem, unsigned long long bDesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
                 ::"r"(dTmem), "r"(aTmem), "l"(bDesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
                 : "memory");
}
// The same MMA issued by a whole warp in uniform control flow: one lane, chosen by elect.sync,
// issues it, so the operands stay warp-uniform. No disable-output-lane mask (every lane of D is
// written); the instruction descriptor is a compile-time constant.
template <uint32_t IDESC>
__device__ __forceinline__ void mmaTf32TsElected(uint32_t dTmem, uint32_t aTmem, unsigned long long bDesc,
                                                 uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred e, p;\n\t"
                 "elect.sync _|e, 0xffffffff;\n\t"
                 "setp.ne.b32 p, %3, 0;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %4, p;\n\t}"
                 ::"r"(dTmem), "r"(aTmem), "l"(bDesc), "r"(accumulate), "n"(IDESC)
                 : "memory");
}
// The 8 MMAs of one full chunk for one 128-feature slice, issued by one elected lane of a warp in
// uniform control flow: MMA p reads A columns aTmem + ASTEP * p and the B tile at descriptor
// bDesc + BSTEP * p, all accumulating into dTmem; the first overwrites D unless
// accumulateFirst != 0. One elect and the operand offsets in one block, so the issuing lane
// does not rebuild each operand between MMAs.
template <uint32_t IDESC, uint32_t ASTEP, uint32_t BSTEP>
__device__ __forceinline__ void mmaTf32Chunk8Elected(uint32_t dTmem, uint32_t aTmem, unsigned long long bDesc,
                                                     uint32_t accumulateFirst) {
    asm volatile("{\n\t.reg .pred e, p, t;\n\t.reg .b32 a<8>;\n\t.reg .b64 b<8>;\n\t"
                 "elect.sync _|e, 0xffffffff;\n\t"
                 "setp.ne.b32 p, %3, 0;\n\t"
                 "setp.ne.b32 t, %4, 0;\n\t"
                 "add.u32 a1, %1, %6;\n\tadd.u32 a2, a1, %6;\n\tadd.u32 a3, a2, %6;\n\t"
                 "add.u32 a4, a3, %6;\n\tadd.u32 a5, a4, %6;\n\tadd.u32 a6, a5, %6;\n\tadd.u32 a7, a6, %6;\n\t"
                 "add.u64 b1, %2, %7;\n\tadd.u64 b2, b1, %7;\n\tadd.u64 b3, b2, %7;\n\t"
                 "add.u64 b4, b3, %7;\n\tadd.u64 b5, b4, %7;\n\tadd.u64 b6, b5, %7;\n\tadd.u64 b7, b6, %7;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %5, p;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [a1], b1, %5, t;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [a2], b2, %5, t;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [a3], b3, %5, t;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [a4], b4, %5, t;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [a5], b5, %5, t;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [a6], b6, %5, t;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [a7], b7, %5, t;\n\t}"
                 ::"r"(dTmem), "r"(aTmem), "l"(bDesc), "r"(accumulateFirst), "r"(1u), "n"(IDESC), "n"(ASTEP),
                 "n"(static_cast<unsigned long long>(BSTEP))
                 : "memory");
}
// tcgen05.commit issued by one elected lane of a warp in uniform control flow.
__device__ __forceinline__ void tcCommitElected(uint32_t bar) {
    asm volatile("{\n\t.reg .pred e;\n\t"
                 "elect.sync _|e, 0xffffffff;\n\t"
                 "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}"
                 ::"r"(bar)
                 : "memory");
}

// Arrive once on the mbarrier when every tcgen05 operation this thread issued so far is done.
__device__ __forceinline__ void tcCommit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// Ticket of the in-kernel merge: atomically increments *counter, wrapping to 0 after
// `bound` (so the last of bound+1 arrivals resets it), with acquire-release ordering at GPU
// scope. Same primitive as the reference (src/kernel/spmm_kernel.cuh:257-260).
__device__ __forceinline__ uint32_t ticketIncrement(uint32_t* counter, uint32_t bound) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;" : "=r"(old) : "l"(counter), "r"(bound) : "memory");
    return old;
}

} // namespace dev
} // namespace tcc
