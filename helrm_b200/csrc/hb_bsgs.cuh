// hb_bsgs.cu -- the fused baby-step + diagonal-MAC kernel of the
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
// (digits D, c0, inner sums) streams once per ciphertext.  Residues below
// 2^40 (the 36-bit q limbs) multiply with the split-30 form, four 32-bit
// multiply-adds per product; the 60-bit special-prime limbs use 64x64->128
// products.  Accumulation is lazy: one modular reduction per output.
// Included by hb_kernels.cu (it reads the per-prime __constant__ table).
#pragma once

namespace hb {

namespace {

constexpr int kThreads = HB_GCH * HB_BT;  // 256: half a warp per giant slot

__device__ __forceinline__ void mac_split_packed(Split3 &s, u64 a_packed, u64 b_packed) {
    split_mac(s, (unsigned)a_packed, (unsigned)(a_packed >> 32), (unsigned)b_packed, (unsigned)(b_packed >> 32));
}

}  // namespace

// NBF = HB_BCH: a full chunk, the baby count is a compile-time constant and
// the unrolled loops carry no guards; NBF = 0: the count is read at run time.
template <int NBF>
__global__ void __launch_bounds__(kThreads, 2)
    k_bsgs_mac(u64 *__restrict__ inner, const u64 *__restrict__ ct, const u64 *__restrict__ D, BsgsChunk ch, int nq,
               int K, int L, int beta, int keyP, int pt_nq, const u64 *__restrict__ pmod_q, int logN, int nbatch,
               size_t ct_stride, size_t d_stride, size_t inner_stride) {
    extern __shared__ u64 sm[];
    const int N = 1 << logN;
    const int e = blockIdx.y;
    const int n0 = blockIdx.x * HB_BT;
    const int ne = nq + K;
    const int p = e < nq ? e : L + (e - nq);
    const PrimeConst pc = c_pc[p];
    const bool fast = pc.q < (1ull << 40);
    const int tid = threadIdx.x;
    const int nb = NBF ? NBF : ch.nbabies;

    // shared memory: descriptors | key tiles [nb][beta][2][BT] | R [nb][2][BT]
    BabyDesc *sdesc = reinterpret_cast<BabyDesc *>(sm);
    u64 *skey = sm + (size_t)HB_BCH * (sizeof(BabyDesc) / 8);
    u64 *sR = skey + (size_t)HB_BCH * beta * 2 * HB_BT;

    for (int i = tid; i < nb * (int)(sizeof(BabyDesc) / 8); i += kThreads)
        sm[i] = reinterpret_cast<const u64 *>(ch.babies)[i];
    __syncthreads();
    // key tiles (split form on fast limbs)
    {
        const int per = beta * 2 * HB_BT;
        for (int i = tid; i < nb * per; i += kThreads) {
            const int bb = i / per, r = i % per, jp = r / HB_BT, n = r % HB_BT;
            const u64 *key = sdesc[bb].key;
            u64 v = 0;
            if (key) v = key[((size_t)jp * keyP + p) * N + n0 + n];
            skey[i] = fast ? split_pack(v) : v;
        }
    }
    // plaintexts of (giant slot gi, baby bb) at this thread's coefficient
    const int gi = tid / HB_BT, nl = tid % HB_BT;
    const bool gactive = gi < ch.gcount;
    const size_t pt_off = ((size_t)(e < nq ? e : pt_nq + (e - nq)) << logN) + n0 + nl;
    u64 ptv[HB_BCH];
#pragma unroll
    for (int bb = 0; bb < HB_BCH; bb++) {
        u64 v = 0;
        if (bb < nb && gactive) {
            const u64 *pp = sdesc[bb].pt[gi];
            if (pp) v = pp[pt_off];
        }
        ptv[bb] = fast ? split_pack(v) : v;
    }
    u64 pq_packed = 0, pq = 0;
    if (e < nq) {
        pq = pmod_q[e];
        pq_packed = split_pack(pq);
    }
    __syncthreads();

    // 32-bit element offsets inside one ciphertext's digits / c0 (the whole
    // extended digit stack of one ciphertext stays far below 2^32 words)
    const unsigned dstride = (unsigned)ne << logN;
    const unsigned erow = (unsigned)e << logN;
    const size_t nall = (size_t)ne << logN;
    for (int b = 0; b < nbatch; b++) {
        const u64 *c0 = ct + b * ct_stride;
        const u64 *c1 = c0 + ((size_t)nq << logN);
        const u64 *Dbe = D + b * d_stride + erow;
        // ---- phase A: baby rotations of this tile.  The gathers of an item
        // (beta digits at the rotated index, and c0) are all issued before
        // any of them is used, so their latencies overlap.
#pragma unroll
        for (int it0 = 0; it0 < (NBF ? NBF * HB_BT : HB_BCH * HB_BT); it0 += kThreads) {
            const int it = it0 + tid;
            if (!NBF && it >= nb * HB_BT) break;
            const int bb = it / HB_BT, n = it % HB_BT;
            const unsigned t = (unsigned)(n0 + n);
            const BabyDesc &bd = sdesc[bb];
            u64 rb, ra;
            if (bd.key == nullptr) {
                rb = e < nq ? mul_mod(pq, c0[erow + t], pc) : 0;
                ra = e < nq ? mul_mod(pq, c1[erow + t], pc) : 0;
            } else {
                const unsigned src = aut_index(t, bd.galois, logN);
                const u64 *kt = skey + (size_t)bb * beta * 2 * HB_BT + n;
                u64 dv[HB_MAX_BETA];
#pragma unroll
                for (int j = 0; j < HB_MAX_BETA; j++)
                    if (j < beta) dv[j] = Dbe[(unsigned)j * dstride + src];
                const u64 cv = e < nq ? c0[erow + src] : 0;
                if (fast) {
                    Split3 sb = {0, 0, 0}, sa = {0, 0, 0};
#pragma unroll
                    for (int j = 0; j < HB_MAX_BETA; j++)
                        if (j < beta) {
                            const u64 d = split_pack(dv[j]);
                            mac_split_packed(sb, d, kt[(j * 2 + 0) * HB_BT]);
                            mac_split_packed(sa, d, kt[(j * 2 + 1) * HB_BT]);
                        }
                    if (e < nq) mac_split_packed(sb, pq_packed, split_pack(cv));
                    rb = split_reduce(sb, pc);
                    ra = split_reduce(sa, pc);
                } else {
                    u128 sb = {0, 0}, sa = {0, 0};
#pragma unroll
                    for (int j = 0; j < HB_MAX_BETA; j++)
                        if (j < beta) {
                            mac128(sb, dv[j], kt[(j * 2 + 0) * HB_BT]);
                            mac128(sa, dv[j], kt[(j * 2 + 1) * HB_BT]);
                        }
                    if (e < nq) mac128(sb, pq, cv);
                    rb = reduce128(sb, pc);
                    ra = reduce128(sa, pc);
                }
            }
            sR[(bb * 2 + 0) * HB_BT + n] = fast ? split_pack(rb) : rb;
            sR[(bb * 2 + 1) * HB_BT + n] = fast ? split_pack(ra) : ra;
        }
        __syncthreads();
        // ---- phase B: inner[g] += pt(g, b) * R_b.  Split sums: S0 takes 16
        // terms below 2^60 before it is normalised (exact, three
        // instructions); one reduction per output.  128-bit sums of at most
        // 32 products below 2^122 need no intermediate reduction.
        if (gactive) {
            u64 vb, va;
            if (fast) {
                Split3 ab = {0, 0, 0}, aa = {0, 0, 0};
#pragma unroll
                for (int bb = 0; bb < HB_BCH; bb++) {
                    if (NBF || bb < nb) {
                        mac_split_packed(ab, ptv[bb], sR[(bb * 2 + 0) * HB_BT + nl]);
                        mac_split_packed(aa, ptv[bb], sR[(bb * 2 + 1) * HB_BT + nl]);
                        if (bb == 15) {
                            split_normalize(ab);
                            split_normalize(aa);
                        }
                    }
                }
                vb = split_reduce(ab, pc);
                va = split_reduce(aa, pc);
            } else {
                u128 ab = {0, 0}, aa = {0, 0};
#pragma unroll
                for (int bb = 0; bb < HB_BCH; bb++) {
                    if (NBF || bb < nb) {
                        mac128(ab, ptv[bb], sR[(bb * 2 + 0) * HB_BT + nl]);
                        mac128(aa, ptv[bb], sR[(bb * 2 + 1) * HB_BT + nl]);
                    }
                }
                vb = reduce128(ab, pc);
                va = reduce128(aa, pc);
            }
            u64 *o = inner + b * inner_stride + (size_t)(ch.gbase + gi) * 2 * nall + erow + n0 + nl;
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
