// gemv_tma.cuh — the TMA-streamed mat-vec: the HBM-bound form of gemv_kernel for rows whose fields are whole
// 16-byte lines (Q8_0 / Q4_K with K % 256 == 0, Q6_K with K % 2048 == 0, BF16 with K % 8 == 0).
//
// Each CTA owns a contiguous slice of rows. One producer warp streams that slice through a ring of shared-memory
// stages with bulk asynchronous copies (cp.async.bulk, one per field per stage, no multicast), each stage tracked by
// an mbarrier's transaction count; 8 or 16 consumer warps stage the activations, then reduce each landed row from
// shared memory and hand the stage back. The producer issues its first stages before griddepcontrol.wait: weights
// depend on nothing, so in a chain of products (a decode step) a product's whole weight slice is in flight while
// the previous product finishes, and the memory system sees every byte of the slice requested at once.
// Every wait is bounded (mbar_wait): one that gives up sets B200_DEVERR_TIMEOUT and the CTA stops consuming.
#pragma once

#include "gemv.cuh"

namespace b200 {

constexpr int kTmaConsumerWarps = 8;
constexpr int kTmaThreads = 32 * (kTmaConsumerWarps + 1);
constexpr unsigned kDevErrTimeout = 4u;  // B200_DEVERR_TIMEOUT

template <class T>
__host__ __device__ inline int64_t tma_row_bytes(int64_t K) {
    int64_t b = 0;
    for (int i = 0; i < T::kFields; i++) b += T::field_row_bytes(K, i);
    return b;
}

template <class T>
__host__ __device__ inline bool tma_fits(int64_t K) {
    for (int i = 0; i < T::kFields; i++)
        if (T::field_row_bytes(K, i) % 16 != 0 || T::field_row_bytes(K, i) == 0) return false;
    return true;
}

// Shared memory: [ring: stages x stage bytes][activation staging][2 x stages mbarriers]
template <class T, int NC>
__host__ __device__ inline size_t tma_smem_bytes(int wtype, int64_t K, int rows_per_stage, int stages) {
    const size_t ring = (size_t) stages * rows_per_stage * tma_row_bytes<T>(K);
    return ring + ((act_smem_bytes(wtype, K, NC) + 15) & ~(size_t) 15) + 16 * (size_t) stages + 16;
}

// Single-column products of `rows` landed rows (field pointers f, row j at local index j). A warp works on 32 / LPR
// rows at once, LPR lanes per row, each lane taking every LPR-th unit of its row (independent units: their loads and
// dp4a chains overlap), then an LPR-lane reduction. LPR = 8 for rows of up to 64 units, else 32. store(j, value).
template <class T, int LPR, class Store>
__device__ __forceinline__ void smem_rows_lpr(const uint8_t * const * f, int64_t K, int rows, const Act & a, const WeightView & w,
                                              int warp, int nwarps, Store store) {
    const int lane = threadIdx.x & 31;
    const int upr = (int) T::units_per_row(K);
    constexpr int kRowsPerPass = 32 / LPR;
    const int sub = lane / LPR, li = lane % LPR;
    for (int j0 = warp * kRowsPerPass; j0 < rows; j0 += nwarps * kRowsPerPass) {
        const int j = j0 + sub;
        const bool row_ok = j < rows;
        double acc[1] = {0.0};
        constexpr int kU = T::kSmemUnroll;
        for (int u0 = 0; u0 < upr; u0 += LPR * kU) {
            typename T::Unit U[kU];
#pragma unroll
            for (int t = 0; t < kU; t++) {
                const int u = u0 + t * LPR + li;
                if (row_ok && u < upr) U[t] = T::load_s(f, K, j, u);
                else U[t] = T::load(w, 0, 0, false);
            }
#pragma unroll
            for (int t = 0; t < kU; t++) {
                const int u = u0 + t * LPR + li;
                T::template dot<1>(U[t], u, row_ok && u < upr, a, acc, nullptr);
            }
        }
        double v = acc[0];
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (row_ok && li == 0) store(j, __double2float_rn(v));
    }
}

// dp4a of unsigned bytes (a) with signed bytes (b), accumulating into c.
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Bits [pos, pos + len) of v (len 0: zero).
__device__ __forceinline__ unsigned bfe_u32(unsigned v, unsigned pos, unsigned len) {
    unsigned d;
    asm("bfe.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(v), "r"(pos), "r"(len));
    return d;
}

// Q4_K rows from shared memory, single column, by 32-byte chunks: 16 lanes per row, two rows per warp pass. Lane li
// of a row takes chunk g = li % 4 of the super-blocks sb = e, e + 4, ... (e = li / 4): the chunk's low nibbles are the
// 32 values of sub-block 2g and its high nibbles those of sub-block 2g + 1, so a lane forms both sub-blocks' exact int32
// sums (dp4a; high nibbles masked in place, their sum a multiple of 16 shifted down exactly), applies their 6-bit scales
// and mins as integers (ggml's sumi and summ restricted to the chunk), then one float32 step with the super-block's
// dx * d and dx * dmin. Each chunk is read as two 16-byte halves, odd super-blocks' lanes taking the second half
// first, and lanes with g >= 2 read the high sub-block's activations first: every 128-bit shared load of an 8-lane
// phase then touches 32 distinct banks.
template <class Store>
__device__ __forceinline__ void smem_rows_q4k(const uint8_t * const * f, int64_t K, int rows, const Act & a, int warp,
                                              int nwarps, Store store) {
    const int lane = threadIdx.x & 31;
    const int sub = lane >> 4, li = lane & 15, g = li & 3, e = li >> 2, h1 = e & 1, h2 = h1 ^ 1;
    const int nsb = (int) (K / 256);
    const bool swap = g >= 2;  // this lane reads the high sub-block's activations first
    const unsigned maskA = swap ? 0xF0F0F0F0u : 0x0F0F0F0Fu, maskB = ~maskA;
    const int xoA = 64 * g + (swap ? 32 : 0), xoB = 64 * g + (swap ? 0 : 32);
    // 6-bit scale / min of sub-blocks 2g and 2g + 1 from meta words y (scale bytes 0..3), z (4..7), w (8..11):
    // j < 4: byte j of y / z; j >= 4: low four bits from byte j - 4 of w (scale: low nibble, min: high nibble), top
    // two bits from bits 6..7 of byte j - 4 of y / z
    const unsigned sh0 = 8u * (unsigned) ((2 * g) & 3), sh1 = sh0 + 8u;
    const unsigned lenlo = swap ? 4u : 6u, himask = swap ? 0x30u : 0u;
    for (int j0 = warp * 2; j0 < rows; j0 += nwarps * 2) {
        const int j = j0 + sub;
        double acc = 0.0;
        if (j < rows) {
            const uint8_t * qr = f[0] + (size_t) j * (size_t) (K / 2) + 32 * g;
            const int4 * mr = reinterpret_cast<const int4 *>(f[1]) + (size_t) j * nsb;
#pragma unroll 2
            for (int sb = e; sb < nsb; sb += 4) {
                const uint8_t * q = qr + 128 * sb;
                const int8_t * xs = a.q + 256 * sb;
                const int4 w1 = *reinterpret_cast<const int4 *>(q + 16 * h1);
                const int4 w2 = *reinterpret_cast<const int4 *>(q + 16 * h2);
                const int4 a1 = *reinterpret_cast<const int4 *>(xs + xoA + 16 * h1);
                const int4 b1 = *reinterpret_cast<const int4 *>(xs + xoB + 16 * h1);
                const int4 a2 = *reinterpret_cast<const int4 *>(xs + xoA + 16 * h2);
                const int4 b2 = *reinterpret_cast<const int4 *>(xs + xoB + 16 * h2);
                const int4 m = mr[sb];
                const int * bs2 = reinterpret_cast<const int *>(a.bs + 16 * sb);
                const int p0 = bs2[2 * g], p1 = bs2[2 * g + 1];  // 16-value sums of sub-blocks 2g and 2g + 1, in pairs
                const float dx = a.d[sb];
                int sA = dp4a_us((unsigned) w1.x & maskA, a1.x, 0);
                int sB = dp4a_us((unsigned) w1.x & maskB, b1.x, 0);
                sA = dp4a_us((unsigned) w1.y & maskA, a1.y, sA);
                sB = dp4a_us((unsigned) w1.y & maskB, b1.y, sB);
                sA = dp4a_us((unsigned) w1.z & maskA, a1.z, sA);
                sB = dp4a_us((unsigned) w1.z & maskB, b1.z, sB);
                sA = dp4a_us((unsigned) w1.w & maskA, a1.w, sA);
                sB = dp4a_us((unsigned) w1.w & maskB, b1.w, sB);
                sA = dp4a_us((unsigned) w2.x & maskA, a2.x, sA);
                sB = dp4a_us((unsigned) w2.x & maskB, b2.x, sB);
                sA = dp4a_us((unsigned) w2.y & maskA, a2.y, sA);
                sB = dp4a_us((unsigned) w2.y & maskB, b2.y, sB);
                sA = dp4a_us((unsigned) w2.z & maskA, a2.z, sA);
                sB = dp4a_us((unsigned) w2.z & maskB, b2.z, sB);
                sA = dp4a_us((unsigned) w2.w & maskA, a2.w, sA);
                sB = dp4a_us((unsigned) w2.w & maskB, b2.w, sB);
                const int il = swap ? sB : sA;
                const int ih = (swap ? sA : sB) >> 4;  // exact: every term of the high-nibble sum is a multiple of 16
                const unsigned my = (unsigned) m.y, mz = (unsigned) m.z, mw = (unsigned) m.w;
                const unsigned srcs = swap ? mw : my, srcm = swap ? (mw >> 4) : mz;
                const int sc0 = (int) (bfe_u32(srcs, sh0, lenlo) | ((my >> (sh0 + 2u)) & himask));
                const int sc1 = (int) (bfe_u32(srcs, sh1, lenlo) | ((my >> (sh1 + 2u)) & himask));
                const int mn0 = (int) (bfe_u32(srcm, sh0, lenlo) | ((mz >> (sh0 + 2u)) & himask));
                const int mn1 = (int) (bfe_u32(srcm, sh1, lenlo) | ((mz >> (sh1 + 2u)) & himask));
                const int si = sc0 * il + sc1 * ih;
                const int sm = mn0 * ((int) (int16_t) (p0 & 0xFFFF) + (p0 >> 16)) + mn1 * ((int) (int16_t) (p1 & 0xFFFF) + (p1 >> 16));
                const float dw = __half2float(__ushort_as_half((unsigned short) ((unsigned) m.x & 0xFFFFu)));
                const float dmw = __half2float(__ushort_as_half((unsigned short) ((unsigned) m.x >> 16)));
                acc = acc_term(acc, __fmul_rn(dx, dw), si);
                acc = acc_term(acc, -__fmul_rn(dx, dmw), sm);
            }
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (j < rows && li == 0) store(j, __double2float_rn(acc));
    }
}

// Q6_K rows from shared memory, single column: LPR lanes per pair of rows; lane li takes the units u = li, li + LPR, ...
// of both rows, unit u being a quarter of super-block sb = u / 4: half hh and values l in [lq, lq + 16) of that half
// (ggml's layout: quant bytes ql[64 hh + l] and ql[64 hh + 32 + l] hold values 128 hh + 32 t + l for t = 0, 2 (low,
// high nibble) and t = 1, 3; bits 2t, 2t + 1 of qh[32 hh + l] are their top bits). The unit's activations are read
// once for both rows (shared memory bandwidth bounds this form). The four 16-value groups t of a unit are visited in
// the order t = k ^ (sb % 2 + 2 hh), k = 0..3, and odd super-blocks load their t-odd quant bytes first: so the 8
// lanes of every 128-bit shared-memory phase (two super-blocks) touch 8 distinct 16-byte bank groups, for the
// activations as for the weights. Per group the int32 sum is exact, sum (q - 32) x = sum q x - 32 bsum, times the
// group's int8 scale; per unit one float32 scale d * dx (as in gemv's unit). Each row's terms are added in the same
// order as with one row per lane.
template <int LPR, class Store>
__device__ __forceinline__ void smem_rows_q6k(const uint8_t * const * f, int64_t K, int rows, const Act & a, int warp,
                                              int nwarps, Store store) {
    const int lane = threadIdx.x & 31;
    constexpr int kPairsPerPass = 32 / LPR;
    const int sub = lane / LPR, li = lane % LPR;
    const int nsb = (int) (K / 256), upr = 4 * nsb;
    const int hh = (li >> 1) & 1, lb = li & 1, sbpar = (li >> 2) & 1;  // LPR is a multiple of 8: fixed per lane
    const int tx = sbpar | (hh << 1);
    const int offP = 64 * hh + 16 * lb + (sbpar ? 32 : 0), offQ = 64 * hh + 16 * lb + (sbpar ? 0 : 32);
    for (int j0 = warp * 2 * kPairsPerPass; j0 < rows; j0 += nwarps * 2 * kPairsPerPass) {
        const int ja = j0 + 2 * sub, jb = ja + 1;
        double acca = 0.0, accb = 0.0;
        if (ja < rows) {
            const int jr = jb < rows ? jb : ja;  // a lone last row computes itself twice and stores once
            const uint8_t * qla = f[0] + (size_t) ja * (size_t) (K / 2);
            const uint8_t * qlb = f[0] + (size_t) jr * (size_t) (K / 2);
            const uint8_t * qha = f[1] + (size_t) ja * (size_t) (K / 4) + 32 * hh + 16 * lb;
            const uint8_t * qhb = f[1] + (size_t) jr * (size_t) (K / 4) + 32 * hh + 16 * lb;
            const int8_t * sca = reinterpret_cast<const int8_t *>(f[2]) + (size_t) ja * nsb * 16 + 8 * hh + lb;
            const int8_t * scb = reinterpret_cast<const int8_t *>(f[2]) + (size_t) jr * nsb * 16 + 8 * hh + lb;
            const uint16_t * dra = reinterpret_cast<const uint16_t *>(f[3]) + (size_t) ja * nsb;
            const uint16_t * drb = reinterpret_cast<const uint16_t *>(f[3]) + (size_t) jr * nsb;
            for (int u = li; u < upr; u += LPR) {
                const int sb = u >> 2;
                const int4 Pa = *reinterpret_cast<const int4 *>(qla + 128 * sb + offP);  // the t with t % 2 == sb % 2
                const int4 Qa = *reinterpret_cast<const int4 *>(qla + 128 * sb + offQ);
                const int4 Ha = *reinterpret_cast<const int4 *>(qha + 64 * sb);
                const int4 Pb = *reinterpret_cast<const int4 *>(qlb + 128 * sb + offP);
                const int4 Qb = *reinterpret_cast<const int4 *>(qlb + 128 * sb + offQ);
                const int4 Hb = *reinterpret_cast<const int4 *>(qhb + 64 * sb);
                const int8_t * xq = a.q + 256 * sb + 128 * hh + 16 * lb;
                const int16_t * bs = a.bs + 16 * sb + 8 * hh + lb;
                int sia = 0, sib = 0;
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int t = k ^ tx;
                    const int ns = 4 * (t >> 1), hs = 2 * t;
                    const int4 xv = *reinterpret_cast<const int4 *>(xq + 32 * t);
                    const int bsum = 32 * (int) bs[2 * t];
                    {
                        const int4 src = (k & 1) ? Qa : Pa;
                        int s = __dp4a((int) ((((unsigned) src.x >> ns) & 0x0F0F0F0Fu) | ((((unsigned) Ha.x >> hs) & 0x03030303u) << 4)), xv.x, 0);
                        s = __dp4a((int) ((((unsigned) src.y >> ns) & 0x0F0F0F0Fu) | ((((unsigned) Ha.y >> hs) & 0x03030303u) << 4)), xv.y, s);
                        s = __dp4a((int) ((((unsigned) src.z >> ns) & 0x0F0F0F0Fu) | ((((unsigned) Ha.z >> hs) & 0x03030303u) << 4)), xv.z, s);
                        s = __dp4a((int) ((((unsigned) src.w >> ns) & 0x0F0F0F0Fu) | ((((unsigned) Ha.w >> hs) & 0x03030303u) << 4)), xv.w, s);
                        sia += (int) sca[16 * sb + 2 * t] * (s - bsum);
                    }
                    {
                        const int4 src = (k & 1) ? Qb : Pb;
                        int s = __dp4a((int) ((((unsigned) src.x >> ns) & 0x0F0F0F0Fu) | ((((unsigned) Hb.x >> hs) & 0x03030303u) << 4)), xv.x, 0);
                        s = __dp4a((int) ((((unsigned) src.y >> ns) & 0x0F0F0F0Fu) | ((((unsigned) Hb.y >> hs) & 0x03030303u) << 4)), xv.y, s);
                        s = __dp4a((int) ((((unsigned) src.z >> ns) & 0x0F0F0F0Fu) | ((((unsigned) Hb.z >> hs) & 0x03030303u) << 4)), xv.z, s);
                        s = __dp4a((int) ((((unsigned) src.w >> ns) & 0x0F0F0F0Fu) | ((((unsigned) Hb.w >> hs) & 0x03030303u) << 4)), xv.w, s);
                        sib += (int) scb[16 * sb + 2 * t] * (s - bsum);
                    }
                }
                const float dx = a.d[sb];
                acca = acc_term(acca, __fmul_rn(__half2float(__ushort_as_half(dra[sb])), dx), sia);
                accb = acc_term(accb, __fmul_rn(__half2float(__ushort_as_half(drb[sb])), dx), sib);
            }
        }
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) {
            acca += __shfl_xor_sync(0xffffffffu, acca, o);
            accb += __shfl_xor_sync(0xffffffffu, accb, o);
        }
        if (li == 0) {
            if (ja < rows) store(ja, __double2float_rn(acca));
            if (jb < rows) store(jb, __double2float_rn(accb));
        }
    }
}

// Q6_K rows from shared memory, one row per lane group (the form for kernels short of registers): LPR lanes per row; lane li takes the units u = li, li + LPR, ... of its
// row, unit u being a quarter of super-block sb = u / 4: half hh and values l in [lq, lq + 16) of that half (ggml's
// layout: quant bytes ql[64 hh + l] and ql[64 hh + 32 + l] hold values 128 hh + 32 t + l for t = 0, 2 (low, high
// nibble) and t = 1, 3; bits 2t, 2t + 1 of qh[32 hh + l] are their top bits). The four 16-value groups t of a unit are
// visited in the order t = k ^ (sb % 2 + 2 hh), k = 0..3, and odd super-blocks load their t-odd quant bytes first: so
// the 8 lanes of every 128-bit shared-memory phase (two super-blocks) touch 8 distinct 16-byte bank groups, for the
// activations as for the weights. Per group the int32 sum is exact, sum (q - 32) x = sum q x - 32 bsum, times the
// group's int8 scale; per unit one float32 scale d * dx (as in gemv's unit).
template <int LPR, class Store>
__device__ __forceinline__ void smem_rows_q6k_single(const uint8_t * const * f, int64_t K, int rows, const Act & a, int warp,
                                              int nwarps, Store store) {
    const int lane = threadIdx.x & 31;
    constexpr int kRowsPerPass = 32 / LPR;
    const int sub = lane / LPR, li = lane % LPR;
    const int nsb = (int) (K / 256), upr = 4 * nsb;
    const int hh = (li >> 1) & 1, lb = li & 1, sbpar = (li >> 2) & 1;  // LPR is a multiple of 8: fixed per lane
    const int tx = sbpar | (hh << 1);
    const int offP = 64 * hh + 16 * lb + (sbpar ? 32 : 0), offQ = 64 * hh + 16 * lb + (sbpar ? 0 : 32);
    for (int j0 = warp * kRowsPerPass; j0 < rows; j0 += nwarps * kRowsPerPass) {
        const int j = j0 + sub;
        double acc = 0.0;
        if (j < rows) {
            const uint8_t * qlr = f[0] + (size_t) j * (size_t) (K / 2);
            const uint8_t * qhr = f[1] + (size_t) j * (size_t) (K / 4) + 32 * hh + 16 * lb;
            const int8_t * scr = reinterpret_cast<const int8_t *>(f[2]) + (size_t) j * nsb * 16 + 8 * hh + lb;
            const uint16_t * dr = reinterpret_cast<const uint16_t *>(f[3]) + (size_t) j * nsb;
            for (int u = li; u < upr; u += LPR) {
                const int sb = u >> 2;
                const int4 P = *reinterpret_cast<const int4 *>(qlr + 128 * sb + offP);  // the t with t % 2 == sb % 2
                const int4 Q = *reinterpret_cast<const int4 *>(qlr + 128 * sb + offQ);
                const int4 H = *reinterpret_cast<const int4 *>(qhr + 64 * sb);
                const int8_t * xq = a.q + 256 * sb + 128 * hh + 16 * lb;
                const int16_t * bs = a.bs + 16 * sb + 8 * hh + lb;
                const int8_t * sc = scr + 16 * sb;
                int si = 0;
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int t = k ^ tx;
                    const int4 src = (k & 1) ? Q : P;
                    const int ns = 4 * (t >> 1), hs = 2 * t;
                    const int4 xv = *reinterpret_cast<const int4 *>(xq + 32 * t);
                    int s = __dp4a((int) ((((unsigned) src.x >> ns) & 0x0F0F0F0Fu) | ((((unsigned) H.x >> hs) & 0x03030303u) << 4)), xv.x, 0);
                    s = __dp4a((int) ((((unsigned) src.y >> ns) & 0x0F0F0F0Fu) | ((((unsigned) H.y >> hs) & 0x03030303u) << 4)), xv.y, s);
                    s = __dp4a((int) ((((unsigned) src.z >> ns) & 0x0F0F0F0Fu) | ((((unsigned) H.z >> hs) & 0x03030303u) << 4)), xv.z, s);
                    s = __dp4a((int) ((((unsigned) src.w >> ns) & 0x0F0F0F0Fu) | ((((unsigned) H.w >> hs) & 0x03030303u) << 4)), xv.w, s);
                    s -= 32 * (int) bs[2 * t];
                    si += (int) sc[2 * t] * s;
                }
                const float dw = __half2float(__ushort_as_half(dr[sb]));
                acc = acc_term(acc, __fmul_rn(dw, a.d[sb]), si);
            }
        }
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (j < rows && li == 0) store(j, __double2float_rn(acc));
    }
}

// Lanes per row: 8 for rows of up to 64 units (a warp reduces 4 rows at once), 32 for longer rows; Q4_K and Q6_K have
// their own forms. A function of K alone, so a row's summation order does not depend on how rows are chunked (launch
// geometry never changes results). kPairedQ6: Q6_K rows two per lane group (fewer shared-memory reads); the persistent
// decode step, short of registers, takes the single-row form, which adds each row's terms in the same order.
template <class T, bool kPairedQ6 = true, class Store>
__device__ __forceinline__ void smem_rows(const uint8_t * const * f, int64_t K, int rows, const Act & a, const WeightView & w,
                                          int warp, int nwarps, Store store) {
    if constexpr (std::is_same<T, TQ4_K>::value) smem_rows_q4k(f, K, rows, a, warp, nwarps, store);
    else if constexpr (std::is_same<T, TQ6_K>::value && kPairedQ6) {
        if (T::units_per_row(K) <= 64) smem_rows_q6k<8>(f, K, rows, a, warp, nwarps, store);
        else smem_rows_q6k<32>(f, K, rows, a, warp, nwarps, store);
    } else if constexpr (std::is_same<T, TQ6_K>::value) {
        if (T::units_per_row(K) <= 64) smem_rows_q6k_single<8>(f, K, rows, a, warp, nwarps, store);
        else smem_rows_q6k_single<32>(f, K, rows, a, warp, nwarps, store);
    } else if (T::units_per_row(K) <= 64) smem_rows_lpr<T, 8>(f, K, rows, a, w, warp, nwarps, store);
    else smem_rows_lpr<T, 32>(f, K, rows, a, w, warp, nwarps, store);
}

// CW consumer warps: 8 (two CTAs per SM fit, for chains whose next product's CTA should start beside this one) or 16
// (one CTA per SM: twice the warps to hide the reduction's shared-memory and dp4a latencies). Ring slot s belongs to
// the group of CW / 8 warps g = s % 8, which splits each of the slot's chunks by rows.
template <class T, int NC, int CW>
__global__ void __launch_bounds__(32 * (CW + 1), CW == kTmaConsumerWarps ? 2 : 1) gemv_tma_kernel(GemvParams p) {
    static_assert(CW % kTmaConsumerWarps == 0, "consumer warps come in groups of one warp per ring slot owner");
    constexpr int kGroup = CW / kTmaConsumerWarps;  // warps per slot owner
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t K = p.w.K;
    const int rps = p.rows_per_stage, stages = p.stages;
    const int64_t row_bytes = tma_row_bytes<T>(K);
    const int64_t stage_bytes = (int64_t) rps * row_bytes;
    uint8_t * ring = smem;
    uint8_t * act_base = smem + stages * stage_bytes;
    uint64_t * full = reinterpret_cast<uint64_t *>(act_base + ((act_smem_bytes(p.w.type, K, NC) + 15) & ~(size_t) 15));
    uint64_t * empty = full + stages;

    const int64_t r_begin = (int64_t) blockIdx.x * p.rows_per_cta;
    const int64_t r_end = r_begin + p.rows_per_cta < p.N ? r_begin + p.rows_per_cta : p.N;
    const int64_t nrows = r_end > r_begin ? r_end - r_begin : 0;
    const int64_t nchunks = (nrows + rps - 1) / rps;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kGroup);  // released by each warp of the group that consumed it
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == CW) {
        // ---- producer ----
        if (lane == 0) {
            const uint8_t * fb[4] = {p.w.f0, p.w.f1, p.w.f2, p.w.f3};
            int64_t issued = 0;  // chunks whose copies were issued
            for (int64_t c = 0; c < nchunks; c++) {
                const int s = (int) (c % stages);
                const int64_t it = c / stages;
                if (it > 0 && !mbar_wait(&empty[s], (uint32_t) ((it - 1) & 1))) {
                    atomicOr(p.err, kDevErrTimeout);
                    break;
                }
                issued = c + 1;
                const int64_t first = r_begin + c * rps;
                const int64_t rows = nrows - c * rps < rps ? nrows - c * rps : rps;
                mbar_arrive_expect_tx(&full[s], (uint32_t) (rows * row_bytes));
                uint8_t * dst = ring + s * stage_bytes;
                for (int i = 0; i < T::kFields; i++) {
                    const int64_t rb = T::field_row_bytes(K, i);
                    bulk_g2s(dst, fb[i] + (p.row0 + first) * rb, (uint32_t) (rows * rb), &full[s]);
                    dst += (int64_t) rps * rb;
                }
                if (c == 0) pdl_launch_dependents();
            }
            if (nchunks == 0) pdl_launch_dependents();
            // the CTA must not exit while copies it issued still land in its shared memory: wait (bounded) for the
            // last use of every slot. On the normal path they have landed already; after a consumer gave up they
            // may not have, and the CTA then ends only once they did (or once this wait also gives up).
            for (int64_t c = issued > stages ? issued - stages : 0; c < issued; c++)
                if (!mbar_wait(&full[c % stages], (uint32_t) ((c / stages) & 1))) atomicOr(p.err, kDevErrTimeout);
        }
        return;
    }

    // ---- consumers (threads 0 .. 32 CW - 1); the first 256 stage the activations (the same reduction order at
    // every CW, so the consumer count never changes results) ----
    const int nthr = 32 * kTmaConsumerWarps;
    pdl_launch_dependents();
    pdl_wait();
    Act a;
    const int kind = act_kind(p.w.type);
    {
        uint8_t * s = act_base;
        a.K = K;
        a.q = nullptr; a.d = nullptr; a.bs = nullptr; a.b = nullptr;
        if (kind == B200_TYPE_BF16) {
            a.b = reinterpret_cast<__nv_bfloat16 *>(s);
        } else {
            a.q = reinterpret_cast<int8_t *>(s);
            s += ((size_t) NC * K + 15) & ~(size_t) 15;
            a.d = reinterpret_cast<float *>(s);
            if (kind == B200_TYPE_Q8_K) {
                s += (size_t) NC * (K / 256) * 4;
                a.bs = reinterpret_cast<int16_t *>(s);
            }
        }
    }
    const int nc = p.ncols < NC ? p.ncols : NC;
    float * xs = reinterpret_cast<float *>(act_base + act_base_bytes(p.w.type, K, NC));
    if (warp < kTmaConsumerWarps) {
        if (NC == 1 && !p.aq && single_fast(K)) stage_one(p, a, kind, nc > 0 ? column_src(p, 0) : p.x, xs, xs + 2 * K, nthr);
        else stage_activations<NC>(p, a, kind, 0, nc, nthr);
    }
    if constexpr (CW > kTmaConsumerWarps) asm volatile("bar.sync 2, %0;" ::"n"(32 * CW) : "memory");

    const int64_t upr = T::units_per_row(K);
    const int nsums = T::sums_per_row(K);
    // chunk c belongs to warp group c % W (W = min(8, stages); the host makes stages a multiple of W), so every ring
    // slot is consumed by one group, whose warps each wait for the slot's phases strictly in order. A parity wait cannot
    // tell phase n from phase n + 2, but a slot's phase n + 1 needs every warp of its group to have released phase n,
    // so no warp of the group can be more than one phase ahead.
    const int W = stages < kTmaConsumerWarps ? stages : kTmaConsumerWarps;
    const int grp = warp % kTmaConsumerWarps, member = warp / kTmaConsumerWarps;
    for (int64_t c = grp; grp < W && c < nchunks; c += W) {
        const int s = (int) (c % stages);
        if (!mbar_wait(&full[s], (uint32_t) ((c / stages) & 1))) {
            if (lane == 0) atomicOr(p.err, kDevErrTimeout);
            break;
        }
        const int64_t rows = nrows - c * rps < rps ? nrows - c * rps : rps;
        const uint8_t * f[4];
        {
            const uint8_t * b = ring + s * stage_bytes;
            for (int i = 0; i < 4; i++) {
                f[i] = b;
                if (i < T::kFields) b += (int64_t) rps * T::field_row_bytes(K, i);
            }
        }
        const int64_t base = r_begin + c * rps;
        if (NC == 1 && !p.sums) {
            smem_rows<T>(f, K, (int) rows, a, p.w, member, kGroup, [&](int j, float v) {
                if (nc > 0) {
                    const int64_t r = base + j;
                    p.y[r] = p.res ? __fadd_rn(p.res[r], v) : v;
                }
            });
        } else {
            for (int64_t j = member; j < rows; j += kGroup) {
                const int64_t r = base + j;  // output row
                int32_t * sums = p.sums ? p.sums + r * nsums : nullptr;
                double acc[NC];
#pragma unroll
                for (int q = 0; q < NC; q++) acc[q] = 0.0;
                for (int64_t u0 = 0; u0 < upr; u0 += 32) {
                    const int64_t u = u0 + lane;
                    const bool valid = u < upr;
                    typename T::Unit U;
                    if (valid) U = T::load_s(f, K, j, u);
                    else U = T::load(p.w, 0, 0, false);
                    T::template dot<NC>(U, u, valid, a, acc, sums);
                }
#pragma unroll
                for (int q = 0; q < NC; q++) {
                    const float v = __double2float_rn(warp_sum_d(acc[q]));
                    if (lane == 0 && q < nc && !p.sums) {
                        float out = v;
                        if (p.res) out = __fadd_rn(p.res[(int64_t) q * p.ldres + r], v);
                        p.y[(int64_t) q * p.ldy + r] = out;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

}  // namespace b200
