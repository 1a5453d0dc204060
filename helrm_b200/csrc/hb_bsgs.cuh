// hb_bsgs.cuh -- the fused baby-step + diagonal-MAC kernel of the
// double-hoisted BSGS linear transform (the embedding PCMM's hot loop).
//
// For one extended limb e and a tile of HB_BT coefficients, over every
// ciphertext of the batch:
//   phase A  R_b = baby rotation of the input, kept in the PQ basis:
//              R_b.b = P*c0[tau_b] + sum_j D_j[tau_b] key_b[j].b,
//              R_b.a = sum_j D_j[tau_b] key_b[j].a        (b = 0: R = P*c)
//   phase B  inner[g] += pt(g, b) * R_b for every giant slot g of the chunk
// The thread block keeps the evaluation-key tiles of its babies in shared
// memory and each thread its plaintext values in registers, so keys and
// diagonals stream from HBM once per batch while the ciphertext data
// (digits D, c0, inner sums) streams once per ciphertext.  On residues
// below 2^40 (the 36-bit q limbs) phase A runs on the FP64 pipe (exact
// centred products key * digit, summed exactly) and phase B on the integer
// pipe in the Karatsuba split-29 form (two 32x32->64 and one 32-bit
// multiply-add per product), so the two phases use different pipes; the
// 60-bit special-prime limbs use 64x64->128 products.  Accumulation is
// lazy: one modular reduction per output.
// Included by hb_kernels.cu (it reads the per-prime __constant__ table).
#pragma once

namespace hb {

namespace {

constexpr int kThreads = HB_GCH * HB_BT;  // 256: half a warp per giant slot

// 16-byte asynchronous copy global -> shared (bypassing L1), grouped by
// commit and waited for with wait_group.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace

// Shared-memory words of one launch (descriptors, key tiles, R tiles of
// `pair` batch items, two gather buffers, rotation tables).  The
// fixed-shape kernels read the descriptors only while setting up, so they
// keep them in the first R tile's space.
__host__ __device__ inline size_t bsgs_smem_words(int beta, int pair = 1, bool fixed = false) {
    return (fixed ? 0 : (size_t)HB_BCH * (sizeof(BabyDesc) / 8)) + (size_t)HB_BCH * beta * 2 * HB_BT +
           (size_t)pair * HB_BCH * 3 * HB_BT +
           (size_t)2 * HB_BCH * (beta + 1) * HB_BT + (size_t)HB_BCH * HB_BT / 8 + HB_BCH / 2 +
           (size_t)HB_BCH * (beta + 1) * (HB_BT / 2);  // gather descriptors (fixed-shape kernels)
}

// NBF = HB_BCH: a full chunk, the baby count is a compile-time constant and
// the unrolled loops carry no guards; NBF = 0: the count is read at run time.
// BETA > 0 fixes the digit count at compile time (row strides and the
// segment division fold to constants); BETA = 0 reads beta_rt.
// ROWS selects the limb rows of the launch: 0 every row (q rows, then the
// special rows; the product form chosen per row at run time), 1 the q rows
// only, every one below 2^40 (split-29 products), 2 the special rows only,
// every one at or above 2^40 (128-bit products).  Row e of the extended
// basis is blockIdx.y + e0.
//
// PAIR = 2 (fixed-shape kernels, chunks of at most HB_GCH / 2 giant slots):
// two batch items per iteration.  Both gather buffers hold the pair, phase A
// builds both R tiles, and in phase B the upper half of the block's giant
// groups works on the second item, so every thread stays busy when a chunk
// has half the giant slots (bs = 2 x 32 for 512 diagonals).  The next
// pair's gathers are issued after phase A and overlap phase B.
//
// The automorphism X -> X^g maps every aligned tile of 16 coefficients (in
// the bit-reversed NTT order) onto another aligned tile of 16, permuted:
// for t = n0 + i the low 4 bits of t land in the top bits of brv(t), and
// multiplying 2 brv(t) + 1 by g leaves the low logN - 3 bits unchanged by i,
// so the high logN - 4 bits of tau(t) are those of tau(n0).  A baby's
// gathers for a tile are therefore one contiguous 128-byte segment per
// digit row, fetched with asynchronous copies one batch item ahead of the
// arithmetic (double buffer); the in-tile permutation is a table built once.
// Two blocks per SM for the split-row kernels of four digits and the
// generic one; the fixed-shape kernels over mixed rows (and of five to
// seven digits) hold one block per SM and take the registers their threads
// need (at two blocks they spill 152 bytes, and the config-4 forward ran
// 1.2 % slower).
template <int NBF, int BETA, int ROWS, int PAIR = 1>
__global__ void __launch_bounds__(kThreads, ((BETA >= 5 || (ROWS == 0 && BETA != 0)) ? 1 : 2))
    k_bsgs_mac(u64 *__restrict__ inner, const u64 *__restrict__ ct, const u64 *__restrict__ D, BsgsChunk ch, int nq,
               int K, int L, int beta_rt, int keyP, int pt_nq, const u64 *__restrict__ pmod_q, int logN, int nbatch, int e0,
               size_t ct_stride, size_t d_stride, size_t inner_stride) {
    extern __shared__ u64 sm[];
    const int N = 1 << logN;
    const int e = blockIdx.y + e0;
    const bool qrow = ROWS == 1 ? true : ROWS == 2 ? false : e < nq;
    const int n0 = blockIdx.x * HB_BT;
    const int ne = nq + K;
    const int p = qrow ? e : L + (e - nq);
    const PrimeConst pc = c_pc[p];
    const bool fast = ROWS == 1 ? true : ROWS == 2 ? false : pc.q < (1ull << 40);
    const int tid = threadIdx.x;
    const int nb = NBF ? NBF : ch.nbabies;
    const int beta = BETA ? BETA : beta_rt;
    const int R1 = beta + 1;  // gathered rows per baby: beta digits, then c0
    // fixed-shape kernels (full chunk, compile-time digit count): precomputed
    // gather descriptors, and the identity baby handled as a rotated one
    // whose key tile holds P mod q at (row 0, b) and (row 1, a)
    constexpr bool kFixed = NBF != 0 && BETA != 0;
    static_assert(PAIR == 1 || (PAIR == 2 && kFixed), "paired items need the fixed-shape kernel");
    const u64 pq_e = qrow ? pmod_q[e] : 0;

    // shared memory: descriptors | key tiles [nb][beta][2][BT] | R [nb][BT][2]
    // | gathers [2][nb][beta+1][BT] | in-tile offsets [nb][BT] (bytes) |
    // source tile bases [nb]
    constexpr size_t kRW = (size_t)HB_BCH * 3 * HB_BT;  // R tile + digit sums of one item
    static_assert(!kFixed || HB_BCH * (sizeof(BabyDesc) / 8) <= kRW, "descriptors fit in an R tile");
    // fixed shape: [R tiles | keys | ...] with the descriptors in the first R
    // tile until the loop starts; otherwise [descriptors | keys | R tiles | ...]
    BabyDesc *sdesc = reinterpret_cast<BabyDesc *>(sm);
    u64 *sR = kFixed ? sm : sm + (size_t)HB_BCH * (sizeof(BabyDesc) / 8) + (size_t)HB_BCH * beta * 2 * HB_BT;
    u64 *skey = kFixed ? sm + PAIR * kRW : sm + (size_t)HB_BCH * (sizeof(BabyDesc) / 8);
    u64 *sG = kFixed ? skey + (size_t)HB_BCH * beta * 2 * HB_BT : sR + PAIR * kRW;
    unsigned char *soff = reinterpret_cast<unsigned char *>(sG + (size_t)2 * HB_BCH * R1 * HB_BT);
    unsigned *sblk = reinterpret_cast<unsigned *>(soff + HB_BCH * HB_BT);
    u64 *sgd = reinterpret_cast<u64 *>(sblk + HB_BCH);  // gather descriptors [NCH][kThreads]
    const size_t gbuf = (size_t)nb * R1 * HB_BT;

    for (int i = tid; i < nb * (int)(sizeof(BabyDesc) / 8); i += kThreads)
        sm[i] = reinterpret_cast<const u64 *>(ch.babies)[i];
    __syncthreads();
    // rotation tables: tile base of tau(n0) and in-tile offsets
    for (int i = tid; i < nb * HB_BT; i += kThreads) {
        const int bb = i / HB_BT, n = i % HB_BT;
        const u64 g = sdesc[bb].galois;
        const unsigned src = sdesc[bb].key ? aut_index((unsigned)(n0 + n), g, logN) : (unsigned)(n0 + n);
        soff[i] = (unsigned char)(src & (HB_BT - 1));
        if (n == 0) sblk[bb] = src & ~(unsigned)(HB_BT - 1);
    }
    // key tiles (split-29 form on fast limbs)
    {
        const int per = beta * 2 * HB_BT;
        for (int i = tid; i < nb * per; i += kThreads) {
            const int bb = i / per, r = i % per, jp = r / HB_BT, n = r % HB_BT;
            const u64 *key = sdesc[bb].key;
            u64 v = 0;
            if (key) v = key[((size_t)jp * keyP + p) * N + n0 + n];
            else if (kFixed && (jp == 0 || jp == 3)) v = pq_e;
            // limbs below 2^40: the key words as exact doubles (phase A on
            // the FP64 pipe); others as they are (128-bit products)
            skey[i] = fast ? (u64)__double_as_longlong(u64_to_d(v)) : v;
        }
    }
    __syncthreads();

    // 32-bit element offsets inside one ciphertext's digits / c0 (the whole
    // extended digit stack of one ciphertext stays far below 2^32 words)
    const unsigned dstride = (unsigned)ne << logN;
    const unsigned erow = (unsigned)e << logN;
    const size_t nall = (size_t)ne << logN;

    // asynchronous gathers of batch item b into buffer buf: for a rotated
    // baby the beta digit rows and c0 at its source tile, for the identity
    // baby c0 and c1 at the tile itself (rows 0 and 1); c-rows exist only on
    // the q limbs
    // segment s = bb * R1 + r; s / R1 by a reciprocal multiply, exact for
    // s < 2^16 / R1 (at most 32 * 9 segments here)
    const unsigned r1mul = (65536u + (unsigned)R1 - 1u) / (unsigned)R1;
    // Fixed-shape kernels: every thread issues exactly NCH 16-byte copies
    // per batch item, whose source offsets (inside one item's digits or
    // ciphertext) and destinations do not depend on the item.  They are
    // packed once per block into sgd[j][tid]: source word offset (bits
    // 0-31), destination byte offset in the gather buffer (32-47), source is
    // the ciphertext (48), copy wanted (49).  A copy not wanted zero-fills
    // its 16 bytes (the identity baby's unused rows, c-rows on special rows).
    constexpr int NCH = kFixed ? NBF * (BETA + 1) * (HB_BT / 2) / kThreads : 0;
    static_assert(!kFixed || NBF * (BETA + 1) * (HB_BT / 2) % kThreads == 0, "gather chunks per thread");
    if (kFixed) {
#pragma unroll
        for (int j = 0; j < NCH; j++) {
            const int i = tid + j * kThreads;
            const unsigned seg = (unsigned)i >> 3;
            const int bb = (int)((seg * r1mul) >> 16), r = (int)seg - bb * R1, k = i & 7;
            u64 srcw, use_c = 1, want = 1;
            if (sdesc[bb].key == nullptr) {
                want = qrow && r < 2;
                srcw = want ? ((u64)r * nq << logN) + erow + n0 + 2 * k : 0;
            } else if (r < beta) {
                use_c = 0;
                srcw = (u64)r * dstride + erow + sblk[bb] + 2 * k;
            } else {
                want = qrow;
                srcw = want ? (u64)erow + sblk[bb] + 2 * k : 0;
            }
            const u64 dstb = (((u64)bb * R1 + r) * HB_BT + 2 * k) * 8;
            sgd[j * kThreads + tid] = srcw | (dstb << 32) | (use_c << 48) | (want << 49);
        }
        // each thread reads only its own descriptors: no barrier needed
    }
    const unsigned sG_sa = (unsigned)__cvta_generic_to_shared(sG);
    auto issue = [&](int b, int buf) {
        const u64 *c0b = ct + b * ct_stride;
        const u64 *Db = D + b * d_stride;
        if (kFixed) {
            const unsigned gb = sG_sa + (unsigned)(buf * gbuf * 8);
#pragma unroll
            for (int j = 0; j < NCH; j++) {
                const u64 d = sgd[j * kThreads + tid];
                const u64 *src = ((d >> 48) & 1 ? c0b : Db) + (unsigned)d;
                const unsigned sa = gb + ((unsigned)(d >> 32) & 0xFFFFu);
                const unsigned nbytes = (unsigned)((d >> 45) & 16);  // bit 49 -> 16 or 0 bytes read
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(src), "r"(nbytes)
                             : "memory");
            }
            cp_async_commit();
            return;
        }
        u64 *Gb = sG + buf * gbuf;
        const int nchunk = nb * R1 * (HB_BT / 2);
        for (int i = tid; i < nchunk; i += kThreads) {
            const unsigned seg = (unsigned)i >> 3;  // HB_BT / 2 = 8 chunks of 16 bytes per segment
            const int bb = (int)((seg * r1mul) >> 16), r = (int)seg - bb * R1, k = i & 7;
            const u64 *src;
            if (sdesc[bb].key == nullptr) {
                if (!qrow || r >= 2) continue;
                src = c0b + ((size_t)r * nq << logN) + erow + n0;
            } else if (r < beta) {
                src = Db + (size_t)r * dstride + erow + sblk[bb];
            } else {
                if (!qrow) continue;
                src = c0b + erow + sblk[bb];
            }
            cp_async16(Gb + ((size_t)bb * R1 + r) * HB_BT + 2 * k, src + 2 * k);
        }
        cp_async_commit();
    };
    issue(0, 0);

    // plaintexts of (giant slot gi, baby bb) at this thread's coefficient
    const int gi = (tid / HB_BT) % (HB_GCH / PAIR), nl = tid % HB_BT;
    const int sub_t = (tid / HB_BT) / (HB_GCH / PAIR);  // item of the pair this thread accumulates
    const bool gactive = gi < ch.gcount;
    const size_t pt_off = ((size_t)(qrow ? e : pt_nq + (e - nq)) << logN) + n0 + nl;
    u64 ptv[HB_BCH];
#pragma unroll
    for (int bb = 0; bb < HB_BCH; bb++) {
        u64 v = 0;
        if (bb < nb && gactive) {
            const u64 *pp = sdesc[bb].pt[gi];
            if (pp) v = pp[pt_off];
        }
        ptv[bb] = fast ? k29_pack(v) : v;
    }
    const u64 pq = pq_e;
    // phase A on limbs below 2^40: exact centred FP64 products key * digit
    // with the digit's quotient estimate fl(d fl(1/q)) (within 2^-15 of
    // key * d / q, so each |t| <= 0.502 q), nine of them summed exactly
    const double qd = u64_to_d(pc.q);
    const double2 pqw = make_double2(u64_to_d(pq), __dmul_rn(u64_to_d(pq), pc.qinv));

    if (PAIR == 2 && nbatch > 1) issue(1, 1);
    for (int b = 0; b < nbatch; b += PAIR) {
        const bool two = PAIR == 2 && b + 1 < nbatch;
        if (PAIR == 2) {
            cp_async_wait<0>();
        } else if (b + 1 < nbatch) {
            issue(b + 1, (b + 1) & 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        // ---- phase A: baby rotations of this tile, from the gathered rows
        constexpr int kItems = NBF ? NBF * HB_BT : HB_BCH * HB_BT;
#pragma unroll
        for (int it0 = 0; it0 < PAIR * kItems; it0 += kThreads) {
            const int itp = it0 + tid;
            const int sub = PAIR == 2 ? itp / kItems : 0;
            const int it = PAIR == 2 ? itp - sub * kItems : itp;
            if (!NBF && it >= nb * HB_BT) break;
            if (PAIR == 2 && sub == 1 && !two) break;
            const u64 *Gb = sG + (PAIR == 2 ? sub : (b & 1)) * gbuf;
            u64 *sRi = sR + sub * kRW;
            uint2 *sRsi = reinterpret_cast<uint2 *>(sRi + (size_t)HB_BCH * 2 * HB_BT);
            const int bb = it / HB_BT, n = it % HB_BT;
            const u64 *g = Gb + (size_t)bb * R1 * HB_BT;
            u64 rb, ra;
            if (!kFixed && sdesc[bb].key == nullptr) {
                rb = qrow ? mul_mod(pq, g[n], pc) : 0;
                ra = qrow ? mul_mod(pq, g[HB_BT + n], pc) : 0;
            } else {
                const int so = soff[it];
                const u64 *kt = skey + (size_t)bb * beta * 2 * HB_BT + n;
                if (fast) {
                    const double *kd = reinterpret_cast<const double *>(kt);
                    double sb = 0.0, sa = 0.0;
#pragma unroll
                    for (int j = 0; j < HB_MAX_BETA; j++)
                        if (j < beta) {
                            const double dv = u64_to_d(g[j * HB_BT + so]);
                            const double2 w = make_double2(dv, __dmul_rn(dv, pc.qinv));
                            sb = __dadd_rn(sb, mulmod_d(kd[(j * 2 + 0) * HB_BT], w, qd));
                            sa = __dadd_rn(sa, mulmod_d(kd[(j * 2 + 1) * HB_BT], w, qd));
                        }
                    if (qrow) sb = __dadd_rn(sb, mulmod_d(u64_to_d(g[beta * HB_BT + so]), pqw, qd));
                    rb = d_mod_to_u64(sb, qd, pc.qinv);
                    ra = d_mod_to_u64(sa, qd, pc.qinv);
                } else {
                    u128 sb = {0, 0}, sa = {0, 0};
#pragma unroll
                    for (int j = 0; j < HB_MAX_BETA; j++)
                        if (j < beta) {
                            const u64 d = g[j * HB_BT + so];
                            mac128(sb, d, kt[(j * 2 + 0) * HB_BT]);
                            mac128(sa, d, kt[(j * 2 + 1) * HB_BT]);
                        }
                    if (qrow) mac128(sb, pq, g[beta * HB_BT + so]);
                    rb = reduce128(sb, pc);
                    ra = reduce128(sa, pc);
                }
            }
            // R tile interleaved {b, a} per coefficient: one 16-byte read in
            // phase B; on fast limbs also the digit sums lo + hi of both
            if (fast) {
                const u64 pb = k29_pack(rb), pa = k29_pack(ra);
                reinterpret_cast<ulonglong2 *>(sRi)[bb * HB_BT + n] = make_ulonglong2(pb, pa);
                sRsi[bb * HB_BT + n] = make_uint2(k29_sum(pb), k29_sum(pa));
            } else {
                reinterpret_cast<ulonglong2 *>(sRi)[bb * HB_BT + n] = make_ulonglong2(rb, ra);
            }
        }
        __syncthreads();
        if (PAIR == 2) {
            // phase A is done with both gather buffers: the next pair's
            // copies overlap phase B
            if (b + 2 < nbatch) issue(b + 2, 0);
            if (b + 3 < nbatch) issue(b + 3, 1);
        }
        // ---- phase B: inner[g] += pt(g, b) * R_b.  Karatsuba split-29 sums
        // of at most 32 products need no intermediate normalisation; one
        // reduction per output.  128-bit sums of at most 32 products below
        // 2^122 need no intermediate reduction either.
        if (gactive && (PAIR == 1 || sub_t == 0 || two)) {
            const u64 *sRt = sR + sub_t * kRW;
            const ulonglong2 *R2 = reinterpret_cast<const ulonglong2 *>(sRt) + nl;
            const uint4 *R4 = reinterpret_cast<const uint4 *>(sRt) + nl;
            const uint2 *RS = reinterpret_cast<const uint2 *>(sRt + (size_t)HB_BCH * 2 * HB_BT) + nl;
            u64 vb, va;
            if (fast) {
                // the q-row kernel alternates two sets of sums over the
                // babies (half-length dependency chains; the merged sums
                // are the same sums of at most 32 products)
                constexpr bool kTwo = ROWS == 1;
                Kara29 ab = {0, 0, 0}, aa = {0, 0, 0}, ab1 = {0, 0, 0}, aa1 = {0, 0, 0};
#pragma unroll
                for (int bb = 0; bb < HB_BCH; bb++) {
                    if (NBF || bb < nb) {
                        const uint4 r = R4[bb * HB_BT];
                        const uint2 rs = RS[bb * HB_BT];
                        const unsigned pl = (unsigned)ptv[bb], ph = (unsigned)(ptv[bb] >> 32), ps = pl + ph;
                        k29_mac_s((kTwo && (bb & 1)) ? ab1 : ab, r.x, r.y, rs.x, pl, ph, ps);
                        k29_mac_s((kTwo && (bb & 1)) ? aa1 : aa, r.z, r.w, rs.y, pl, ph, ps);
                    }
                }
                if (kTwo) {
                    ab.s0 += ab1.s0, ab.m += ab1.m, ab.s2 += ab1.s2;
                    aa.s0 += aa1.s0, aa.m += aa1.m, aa.s2 += aa1.s2;
                }
                vb = k29_reduce(ab, pc);
                va = k29_reduce(aa, pc);
            } else {
                u128 ab = {0, 0}, aa = {0, 0};
#pragma unroll
                for (int bb = 0; bb < HB_BCH; bb++) {
                    if (NBF || bb < nb) {
                        const ulonglong2 r = R2[bb * HB_BT];
                        mac128(ab, ptv[bb], r.x);
                        mac128(aa, ptv[bb], r.y);
                    }
                }
                vb = reduce128(ab, pc);
                va = reduce128(aa, pc);
            }
            u64 *o = inner + (b + sub_t) * inner_stride + (size_t)(ch.gbase + gi) * 2 * nall + erow + n0 + nl;
            if (ch.accumulate) {
                vb = add_mod(vb, o[0], pc.q);
                va = add_mod(va, o[nall], pc.q);
            }
            o[0] = vb;
            o[nall] = va;
        }
        __syncthreads();
    }
}

}  // namespace hb
