// hb_bsgs_tc.cuh -- the fused baby-step + diagonal-MAC kernel of the
// double-hoisted BSGS linear transform with the plaintext products on the
// 5th-generation tensor cores (tcgen05, int8 MMA, accumulators in TMEM).
//
// The diagonal MAC of one extended limb e at one coefficient n is a small
// matrix product shared by the whole batch:
//     inner[ct][poly][g] = sum_b R_b[ct][poly] * pt(g, b)     (mod q_e)
// with M = ciphertexts x {b, a} polys, K = babies (32), N = giant slots (16).
// Residues below 2^37 are split into five byte planes, x = sum_i x_i 2^(8i);
// the product of two such numbers is sum over shift classes s = i + j
// (0..8) of P_s 2^(8s), P_s = sum_{i+j=s} sum_b a_i[b] b_j[b], an exact
// integer below 5 * 32 * 255^2 < 2^24.  One MMA per A plane i (K = 32
// bytes) against a B window that places plane j = s - i of the plaintext
// in the 16 accumulator columns of class s (zero blocks elsewhere):
//
//   B buffer (16-row blocks):  [0 0 0 0][P0 P1 P2 P3 P4][0 0 0 0] ...
//   A plane i reads the window starting i blocks before P0, 9 blocks (N = 144)
//
// so five MMAs of N = 144 accumulate all nine classes of all 16 giant slots
// in 144 TMEM columns; the epilogue forms sum_s P_s (2^(8s) mod q) exactly
// in 64-bit integers and reduces once.  Every step is exact: the result is
// the residue the CUDA-core kernel (hb_bsgs.cuh) computes, bit for bit.
//
// Phase A (the baby rotations R_b, keys times rotated digits) runs on the
// CUDA cores with exact arithmetic, as in hb_bsgs.cuh.  A CTA handles a
// tile of four coefficients (an aligned 4-tile maps onto an aligned 4-tile
// under every automorphism, so each gather is one 32-byte sector) for 32
// ciphertexts (M = 64 rows); two M = 64 accumulators share 144 columns in
// the two halves of each TMEM lane quadrant (lane offsets 0 and 16).  A
// pass covers 32 ciphertexts; every CTA works on the same limb at a time.
//
// Roles (one CTA per SM, persistent over tiles; 672 threads):
//   warps 0-15  producers: R_b for (baby, coefficient) pairs over a quarter
//               of the pass's ciphertexts each, gathered through a
//               per-thread ring of asynchronous copies and written as byte
//               planes into the A buffer (double-buffered); R.b on the
//               integer pipe (Karatsuba split-29 sums, one reduction), R.a
//               on the FP64 pipe (exact centred products), so the two
//               pipes work side by side
//   warps 16-19 epilogue: TMEM -> registers -> reduction -> staged stores
//   warp 20     MMA issue and the bulk copies of the plaintext planes
// Pipeline hand-offs are mbarriers; every wait is bounded by a clock limit
// and, when it runs out, sets an error word (read on the host at the next
// synchronisation) and makes the whole CTA leave its loops, wait for its
// own copies and MMAs (bounded) and release its TMEM.
// Included by hb_kernels.cu (it reads the per-prime __constant__ table).
#pragma once

namespace hb {

constexpr int kTcCoef = 4;             // coefficients per tile
constexpr int kTcCts = 32;             // ciphertexts per pass (MMA M = 64)
constexpr int kTcPlanes = 5;           // byte planes of a residue below 2^40
constexpr int kTcClasses = 9;          // shift classes of the plane products
constexpr int kTcN = kTcClasses * HB_GCH;  // 144 accumulator columns per coefficient
constexpr int kTcProducers = 512;
constexpr int kTcQuarters = kTcProducers / 128;  // producer groups, each over every 4th ciphertext
constexpr int kTcEpi = 128;
constexpr int kTcThreads = kTcProducers + kTcEpi + 32;
constexpr int kTcAPlane = 64 * 32;                    // 64 rows x 32 babies (K-major core matrices)
constexpr int kTcACoef = kTcPlanes * kTcAPlane + 16;  // +16 B spreads the 4 coefficients over banks
constexpr int kTcABuf = kTcCoef * kTcACoef;
constexpr int kTcBBlock = HB_GCH * 32;                 // 16 giant rows x 32 babies
constexpr int kTcBBlocks = 4 + kTcCoef * (kTcPlanes + 4);
constexpr int kTcBBuf = kTcBBlocks * kTcBBlock;
constexpr int kTcPtTile = kTcCoef * kTcPlanes * kTcBBlock;  // plaintext planes of one tile in HBM
constexpr int kTcStage = kTcCoef * HB_GCH * 64 * 8;
constexpr int kTcRing = 3;  // ciphertexts of gathered words in flight per producer thread
constexpr int kTcGather = kTcRing * 5 * kTcProducers * 8;
constexpr int kTcSmem = 2 * kTcABuf + 2 * kTcBBuf + kTcStage + 128 + kTcGather;
static_assert(kTcABuf % 16 == 0 && kTcBBuf % 1024 == 0, "smem alignment");

namespace tc {

__device__ __forceinline__ unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }

// byte offset of (row, k) in a K-major tile of 32-byte rows without swizzle:
// core matrices of 8 rows x 16 bytes, the two K halves 128 B apart (LBO),
// 8-row groups 256 B apart (SBO)
__device__ __forceinline__ int tile_off(int row, int k) {
    return (row >> 3) * 256 + (k >> 4) * 128 + (row & 7) * 16 + (k & 15);
}
// shared-memory matrix descriptor (tcgen05), no swizzle
__device__ __forceinline__ uint64_t sdesc(unsigned saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) |
           ((uint64_t)1 << 46);
}
// instruction descriptor: s32 accumulator, u8 x u8, both K-major, N = 144, M = 64
constexpr unsigned kIdesc = (2u << 4) | ((unsigned)(kTcN >> 3) << 17) | ((64u >> 4) << 24);

__device__ __forceinline__ void mbar_init(unsigned a, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(unsigned a) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(unsigned a, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(unsigned a, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait for the given phase parity.  Gives up after `limit_ns`, or
// at once when another thread of the CTA has given up (*abort set, unless
// abort is null); returns false then, after recording `code` in *err.
__device__ __forceinline__ bool mbar_wait(unsigned a, unsigned parity, volatile int *abort, int *err, int code,
                                          unsigned long long limit_ns) {
    if (mbar_try(a, parity)) return true;
    const unsigned long long t0 = gtimer();
    for (unsigned it = 1;; it++) {
        if (mbar_try(a, parity)) return true;
        if (abort && *abort) return false;
        if ((it & 63) == 0 && gtimer() - t0 > limit_ns) {
            if (abort) *abort = 1;
            atomicOr(err, code);
            return false;
        }
    }
}
__device__ __forceinline__ void bulk_g2s(unsigned dst, const void *src, unsigned bytes, unsigned mbar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(mbar)
                 : "memory");
}
__device__ __forceinline__ void mma_i8(unsigned tmem_d, uint64_t ad, uint64_t bd, unsigned accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(ad), "l"(bd), "r"(kIdesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void mma_commit(unsigned mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
                 : "memory");
}
__device__ __forceinline__ void tmem_ld8(unsigned taddr, unsigned (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld4(unsigned taddr, unsigned (&v)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void named_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ void cp_async8(u64 *smem, const u64 *gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}

}  // namespace tc

// Error bits of the tensor-core MAC (the device word the host checks).
#define HB_TC_ERR_PRODUCER 1
#define HB_TC_ERR_MMA 2
#define HB_TC_ERR_EPILOGUE 4
#define HB_TC_ERR_DRAIN 8

// inner[ct][gslot][poly][e][n] for the pass's ciphertexts [ct0, ct0 + 32)
// and every q row e < nq.  ptp: the chunk's plaintexts as byte planes,
// [e][tile][coef][plane][16 x 32 canonical tile].  cls: [nq][9] values
// 2^(8s) mod q_e.  BETA digits, every q row below 2^37.
template <int BETA>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_bsgs_mma(u64 *__restrict__ inner, const u64 *__restrict__ ct, const u64 *__restrict__ D, BsgsChunk ch,
               const uint8_t *__restrict__ ptp, const u64 *__restrict__ cls, int nq, int K, int keyP,
               const u64 *__restrict__ pmod_q, int logN, int nbatch, int ct0, size_t ct_stride, size_t d_stride,
               size_t inner_stride, int *err, unsigned long long limit_ns) {
    extern __shared__ __align__(1024) unsigned char smem[];
    unsigned char *sA = smem;                        // [2][kTcABuf]
    unsigned char *sB = smem + 2 * kTcABuf;          // [2][kTcBBuf]
    u64 *sS = reinterpret_cast<u64 *>(sB + 2 * kTcBBuf);  // [coef][giant][row]
    u64 *bars = reinterpret_cast<u64 *>(reinterpret_cast<unsigned char *>(sS) + kTcStage);
    // barriers: fullA[2], emptyA[2], fullB[2], tmem_full, tmem_empty, drain;
    // then the TMEM base address and the abort flag
    unsigned *s_tmem = reinterpret_cast<unsigned *>(bars + 9);
    volatile int *s_abort = reinterpret_cast<volatile int *>(bars + 10);
    u64 *sG = bars + 16;  // producers' gather ring [kTcRing][5][kTcProducers]
    const unsigned b_fullA = tc::smem_u32(bars + 0), b_emptyA = tc::smem_u32(bars + 2);
    const unsigned b_fullB = tc::smem_u32(bars + 4), b_tfull = tc::smem_u32(bars + 6);
    const unsigned b_tempty = tc::smem_u32(bars + 7), b_drain = tc::smem_u32(bars + 8);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int N = 1 << logN;
    const int tpl = N / kTcCoef;  // tiles per limb (a power of two)
    const int tpl_log = logN - 2;
    const long total = (long)nq * tpl;
    const size_t nall = (size_t)(nq + K) << logN;

    if (tid == 0) {
        for (int i = 0; i < 2; i++) {
            tc::mbar_init(b_fullA + 8 * i, kTcProducers / 32);  // one arrival per producer warp
            tc::mbar_init(b_emptyA + 8 * i, 1);
            tc::mbar_init(b_fullB + 8 * i, 1);
        }
        tc::mbar_init(b_tfull, 1);
        tc::mbar_init(b_tempty, 4);  // one arrival per epilogue warp
        tc::mbar_init(b_drain, 1);
        *s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // zero both B buffers once: the bulk copies fill only the plane blocks
    for (int i = tid; i < 2 * kTcBBuf / 16; i += kTcThreads)
        reinterpret_cast<uint4 *>(sB)[i] = make_uint4(0, 0, 0, 0);
    const int kMmaWarp = (kTcProducers + kTcEpi) / 32;
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_u32(s_tmem)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const unsigned tmem = *s_tmem;

    if (warp < kTcProducers / 32) {
        // ---------------------------------------------------------------- producers
        const int quarter = tid >> 7, wl = (tid >> 5) & 3;
        const int bb = 8 * wl + (lane >> 2), c = lane & 3;
        const bool active = bb < ch.nbabies;
        u64 galois = 1;
        const u64 *key = nullptr;
        if (active) {
            galois = ch.babies[bb].galois;
            key = ch.babies[bb].key;
        }
        const unsigned dstride = (unsigned)(nq + K) << logN;  // one digit's rows inside D
        for (long it = 0;; it++) {
            const long tile = blockIdx.x + it * gridDim.x;
            if (tile >= total) break;
            const int buf = (int)(it & 1);
            if (it >= 2 && !tc::mbar_wait(b_emptyA + 8 * buf, (unsigned)(((it >> 1) - 1) & 1), s_abort, err,
                                          HB_TC_ERR_PRODUCER, limit_ns))
                break;
            const int e = (int)(tile >> tpl_log), T = (int)(tile & (tpl - 1));
            const unsigned n = (unsigned)(T * kTcCoef + c);
            const PrimeConst pc = c_pc[e];
            const double qd = u64_to_d(pc.q);
            const u64 pq = pmod_q[e];
            const double2 pqw = make_double2(u64_to_d(pq), __dmul_rn(u64_to_d(pq), pc.qinv));
            const u64 pqk = k29_pack(pq);
            const unsigned erow = (unsigned)e << logN;
            unsigned char *A = sA + buf * kTcABuf + c * kTcACoef;
            if (active) {
                // keys: the b part in split-29 form (integer pipe), the a
                // part as exact doubles (FP64 pipe)
                u64 kbk[BETA];
                double ka[BETA];
                unsigned src = n;
                if (key) {
                    src = aut_index(n, galois, logN);
#pragma unroll
                    for (int j = 0; j < BETA; j++) {
                        kbk[j] = k29_pack(key[((size_t)(j * 2 + 0) * keyP + e) * N + n]);
                        ka[j] = u64_to_d(key[((size_t)(j * 2 + 1) * keyP + e) * N + n]);
                    }
                }
                const int ob = tc::tile_off(0, bb) - tc::tile_off(0, 0);
                int nct = nbatch - ct0;
                if (nct > kTcCts) nct = kTcCts;
                // ciphertexts quarter, quarter + 4, ...
                const int nloc = nct > quarter ? (nct - quarter + kTcQuarters - 1) / kTcQuarters : 0;
                // asynchronous 8-byte copies of this thread's gathered words
                // (BETA digits and c0 at the rotated position; the identity
                // baby: c0 and c1 at n) into its own ring slots: only this
                // thread reads them, so its own wait_group orders them
                auto issue = [&](int k) {
                    const int cg = ct0 + quarter + kTcQuarters * k;
                    const u64 *cb = ct + (size_t)cg * ct_stride;
                    u64 *slot = sG + (size_t)(k % kTcRing) * 5 * kTcProducers + tid;
                    if (key) {
                        const u64 *db = D + (size_t)cg * d_stride + erow + src;
#pragma unroll
                        for (int j = 0; j < BETA; j++) tc::cp_async8(slot + j * kTcProducers, db + (size_t)j * dstride);
                        tc::cp_async8(slot + BETA * kTcProducers, cb + erow + src);
                    } else {
                        tc::cp_async8(slot, cb + erow + n);
                        tc::cp_async8(slot + kTcProducers, cb + ((size_t)nq << logN) + erow + n);
                    }
                };
#pragma unroll
                for (int k = 0; k < kTcRing - 1; k++) {
                    if (k < nloc) issue(k);
                    asm volatile("cp.async.commit_group;" ::: "memory");
                }
                for (int k = 0; k < nloc; k++) {
                    if (k + kTcRing - 1 < nloc) issue(k + kTcRing - 1);
                    asm volatile("cp.async.commit_group;" ::: "memory");
                    asm volatile("cp.async.wait_group %0;" ::"n"(kTcRing - 1) : "memory");
                    const u64 *slot = sG + (size_t)(k % kTcRing) * 5 * kTcProducers + tid;
                    const int ctl = quarter + kTcQuarters * k;
                    u64 rb, ra;
                    if (key) {
                        Kara29 sb = {0, 0, 0};
                        double sa = 0.0;
#pragma unroll
                        for (int j = 0; j < BETA; j++) {
                            const u64 d = slot[j * kTcProducers];
                            const u64 dk = k29_pack(d);
                            k29_mac(sb, kbk[j], dk, k29_sum(dk));
                            const double dv = u64_to_d(d);
                            sa = __dadd_rn(sa, mulmod_d(ka[j], make_double2(dv, __dmul_rn(dv, pc.qinv)), qd));
                        }
                        const u64 c0k = k29_pack(slot[BETA * kTcProducers]);
                        k29_mac(sb, pqk, c0k, k29_sum(c0k));
                        rb = k29_reduce(sb, pc);
                        ra = d_mod_to_u64(sa, qd, pc.qinv);
                    } else {
                        Kara29 sb = {0, 0, 0};
                        const u64 c0k = k29_pack(slot[0]);
                        k29_mac(sb, pqk, c0k, k29_sum(c0k));
                        rb = k29_reduce(sb, pc);
                        ra = d_mod_to_u64(mulmod_d(u64_to_d(slot[kTcProducers]), pqw, qd), qd, pc.qinv);
                    }
                    const int offb = tc::tile_off(ctl, 0) + ob, offa = tc::tile_off(32 + ctl, 0) + ob;
#pragma unroll
                    for (int p = 0; p < kTcPlanes; p++) {
                        A[p * kTcAPlane + offb] = (unsigned char)(rb >> (8 * p));
                        A[p * kTcAPlane + offa] = (unsigned char)(ra >> (8 * p));
                    }
                }
                asm volatile("cp.async.wait_group 0;" ::: "memory");
            }
            // the A planes are read by the tensor cores (async proxy)
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(b_fullA + 8 * buf);
        }
    } else if (warp < kMmaWarp) {
        // ---------------------------------------------------------------- epilogue
        const int quad = warp & 3;  // TMEM lane quadrant this warp may access
        const int et = tid - kTcProducers;  // 0..127
        for (long it = 0;; it++) {
            const long tile = blockIdx.x + it * gridDim.x;
            if (tile >= total) break;
            if (!tc::mbar_wait(b_tfull, (unsigned)(it & 1), s_abort, err, HB_TC_ERR_EPILOGUE, limit_ns)) break;
            tc::fence_after();
            const int e = (int)(tile >> tpl_log), T = (int)(tile & (tpl - 1));
            const PrimeConst pc = c_pc[e];
            unsigned clo[kTcClasses], chi[kTcClasses];
#pragma unroll
            for (int s = 0; s < kTcClasses; s++) {
                const u64 v = cls[(size_t)e * kTcClasses + s];
                clo[s] = (unsigned)v;
                chi[s] = (unsigned)(v >> 32);
            }
            const int m = 16 * quad + (lane & 15);  // accumulator row of this thread
#pragma unroll 1
            for (int part = 0; part < 2 * (HB_GCH / 4); part++) {
                // column slot (a pair of coefficients in the two lane halves)
                // and a group of four giant slots
                const int slot = part / (HB_GCH / 4), g0 = (part % (HB_GCH / 4)) * 4;
                const int cc = 2 * slot + (lane >> 4);
                u64 lo[4];
                unsigned hi[4];
#pragma unroll
                for (int g = 0; g < 4; g++) lo[g] = 0, hi[g] = 0;
                const unsigned ta = tmem + ((unsigned)(32 * quad) << 16) + (unsigned)(kTcN * slot + g0);
                // all nine classes in flight, one wait
                unsigned v[kTcClasses][4];
#pragma unroll
                for (int s = 0; s < kTcClasses; s++) tc::tmem_ld4(ta + 16 * s, v[s]);
                tc::tmem_wait_ld();
#pragma unroll
                for (int s = 0; s < kTcClasses; s++) {
#pragma unroll
                    for (int g = 0; g < 4; g++) {
                        asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(lo[g]) : "r"(v[s][g]), "r"(clo[s]));
                        hi[g] += v[s][g] * chi[s];
                    }
                }
                // x = lo + hi 2^32 < 2^63.2 (P_s < 2^24, 2^(8s) mod q < 2^37):
                // quotient estimate on the FP64 pipe, two conditional fixes
#pragma unroll
                for (int g = 0; g < 4; g++) {
                    const u64 x = lo[g] + ((u64)hi[g] << 32);
                    const double xd = __fma_rn(u32_to_double((unsigned)(x >> 32)), 4294967296.0,
                                               u32_to_double((unsigned)x));
                    const u64 Q = (u64)__double_as_longlong(__fma_rn(xd, pc.qinv, 4503599627370496.0)) &
                                  0x000FFFFFFFFFFFFFull;
                    u64 r = x - Q * pc.q;
                    if ((long long)r < 0) r += pc.q;
                    if (r >= pc.q) r -= pc.q;
                    sS[((size_t)cc * HB_GCH + g0 + g) * 64 + m] = r;
                }
            }
            // TMEM drained: the next tile's MMAs may overwrite it
            tc::fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(b_tempty);
            tc::named_sync(1, kTcEpi);
            // stores: 32 bytes (four coefficients) per (row, giant slot)
            {
                const int r = et >> 1, g0 = (et & 1) * (HB_GCH / 2);
                const int ctl = r & 31, poly = r >> 5, cg = ct0 + ctl;
                if (cg < nbatch) {
                    u64 *obase = inner + (size_t)cg * inner_stride + (size_t)poly * nall + ((size_t)e << logN) +
                                 (size_t)T * kTcCoef;
#pragma unroll 2
                    for (int g = g0; g < g0 + HB_GCH / 2; g++) {
                        if (g >= ch.gcount) break;
                        u64 v0 = sS[((size_t)0 * HB_GCH + g) * 64 + r], v1 = sS[((size_t)1 * HB_GCH + g) * 64 + r];
                        u64 v2 = sS[((size_t)2 * HB_GCH + g) * 64 + r], v3 = sS[((size_t)3 * HB_GCH + g) * 64 + r];
                        ulonglong2 *o = reinterpret_cast<ulonglong2 *>(obase + (size_t)(ch.gbase + g) * 2 * nall);
                        if (ch.accumulate) {
                            const ulonglong2 p0 = o[0], p1 = o[1];
                            v0 = add_mod(v0, p0.x, pc.q), v1 = add_mod(v1, p0.y, pc.q);
                            v2 = add_mod(v2, p1.x, pc.q), v3 = add_mod(v3, p1.y, pc.q);
                        }
                        o[0] = make_ulonglong2(v0, v1);
                        o[1] = make_ulonglong2(v2, v3);
                    }
                }
            }
            tc::named_sync(1, kTcEpi);
        }
    } else {
        // ---------------------------------------------------------------- MMA issue
        if (lane == 0) {
            long it = 0;
            long b_issued = 0, b_waited = 0;  // B loads issued / completed: tiles [0, b_issued) / [0, b_waited)
            // plaintext planes of tile `i` into B buffer i & 1, once its
            // previous contents are consumed (the MMAs of tile i - 2)
            auto load_b = [&](long i) -> bool {
                const long tile = blockIdx.x + i * gridDim.x;
                if (tile >= total) return true;
                const int buf = (int)(i & 1);
                if (i >= 2 && !tc::mbar_wait(b_emptyA + 8 * buf, (unsigned)(((i >> 1) - 1) & 1), s_abort, err,
                                             HB_TC_ERR_MMA, limit_ns))
                    return false;
                const unsigned dst = tc::smem_u32(sB + buf * kTcBBuf);
                const uint8_t *src = ptp + (size_t)tile * kTcPtTile;
                tc::mbar_arrive_tx(b_fullB + 8 * buf, (unsigned)kTcPtTile);
                for (int c = 0; c < kTcCoef; c++)
                    tc::bulk_g2s(dst + (4 + 9 * c) * kTcBBlock, src + c * kTcPlanes * kTcBBlock,
                                 kTcPlanes * kTcBBlock, b_fullB + 8 * buf);
                b_issued = i + 1;
                return true;
            };
            bool ok = load_b(0);
            for (; ok; it++) {
                const long tile = blockIdx.x + it * gridDim.x;
                if (tile >= total) break;
                const int buf = (int)(it & 1);
                if (!(ok = load_b(it + 1))) break;
                if (!tc::mbar_wait(b_fullA + 8 * buf, (unsigned)((it >> 1) & 1), s_abort, err, HB_TC_ERR_MMA,
                                   limit_ns))
                    break;
                if (!tc::mbar_wait(b_fullB + 8 * buf, (unsigned)((it >> 1) & 1), s_abort, err, HB_TC_ERR_MMA,
                                   limit_ns))
                    break;
                b_waited = it + 1;
                if (it >= 1 &&
                    !tc::mbar_wait(b_tempty, (unsigned)((it - 1) & 1), s_abort, err, HB_TC_ERR_MMA, limit_ns))
                    break;
                tc::fence_after();
                const unsigned abase = tc::smem_u32(sA + buf * kTcABuf);
                const unsigned bbase = tc::smem_u32(sB + buf * kTcBBuf);
#pragma unroll
                for (int c = 0; c < kTcCoef; c++) {
                    const unsigned d = tmem + ((unsigned)(16 * (c & 1)) << 16) + (unsigned)(kTcN * (c >> 1));
#pragma unroll
                    for (int j = 0; j < kTcPlanes; j++)
                        tc::mma_i8(d, tc::sdesc(abase + c * kTcACoef + j * kTcAPlane),
                                   tc::sdesc(bbase + (4 + 9 * c - j) * kTcBBlock), j > 0);
                }
                tc::mma_commit(b_emptyA + 8 * buf);
                tc::mma_commit(b_tfull);
            }
            // leave nothing in flight, even after an abort: the bulk copies
            // not yet waited for, then every MMA this thread issued (bounded
            // waits that ignore the abort flag)
            for (long i = b_waited; i < b_issued; i++)
                tc::mbar_wait(b_fullB + 8 * (int)(i & 1), (unsigned)((i >> 1) & 1), nullptr, err, HB_TC_ERR_DRAIN,
                              limit_ns);
            tc::mma_commit(b_drain);
            tc::mbar_wait(b_drain, 0, nullptr, err, HB_TC_ERR_DRAIN, limit_ns);
        }
        __syncwarp();
    }

    // ---------------------------------------------------------------- teardown
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

// Plaintext byte planes of one chunk for the q rows: ptp[e][tile][coef][plane]
// [16 x 32 canonical tile] <- pt(g, b)[e][n]; missing (g, b) pairs are zero.
__global__ void k_pt_planes(uint8_t *__restrict__ ptp, const BabyDesc *__restrict__ babies, int nbabies, int gcount,
                            int logN) {
    const int e = blockIdx.y;
    const int N = 1 << logN;
    const int n = blockIdx.x * blockDim.x + threadIdx.x;  // coefficient
    if (n >= N) return;
    const int T = n / kTcCoef, c = n % kTcCoef;
    uint8_t *dst = ptp + ((size_t)e * (N / kTcCoef) + T) * kTcPtTile + (size_t)c * kTcPlanes * kTcBBlock;
    for (int bb = 0; bb < 32; bb++) {
        for (int g = 0; g < HB_GCH; g++) {
            u64 v = 0;
            if (bb < nbabies && g < gcount) {
                const u64 *p = babies[bb].pt[g];
                if (p) v = p[((size_t)e << logN) + n];
            }
            const int off = (g >> 3) * 256 + (bb >> 4) * 128 + (g & 7) * 16 + (bb & 15);
#pragma unroll
            for (int pl = 0; pl < kTcPlanes; pl++) dst[pl * kTcBBlock + off] = (uint8_t)(v >> (8 * pl));
        }
    }
}

}  // namespace hb
