// hb_kernels.cuh -- device kernels of the B200 CKKS backend and their
// host-side launchers.  Data layout (HBM): a polynomial is a stack of
// limbs, each limb N contiguous uint64 residues in the bit-reversed NTT
// order.  A ciphertext at level l is [2][l+1][N]; an extended-basis (PQ)
// polynomial is [l+1+K][N] with the q rows first and the K special-prime
// rows after them.
#pragma once
#include <cuda_runtime.h>

#include "hb_arith.cuh"

namespace hb {

// Maps row r of a batched launch to its prime index.  Rows come in blocks
// of `per` rows; row e of a block is main prime e when e < nq and special
// prime L + (e - nq) otherwise.  With alpha > 0, rows of block b that
// belong to digit b ([b*alpha, min(b*alpha+alpha, nq))) are skipped (the
// ModUp output keeps the input limbs of its own digit).
struct RowMap {
    int per;
    int nq;
    int L;
    int alpha = 0;   // > 0: skip the rows of the block's own digit
    int ndig = 1;    // digit of block b is (b % ndig)
    int pbase = 0;   // main-prime rows start at prime pbase
    __host__ __device__ int prime(int r) const {
        int e = r % per;
        return e < nq ? pbase + e : L + (e - nq);
    }
    __host__ __device__ bool skip(int r) const {
        if (alpha <= 0) return false;
        int b = (r / per) % ndig, e = r % per;
        int lo = b * alpha, hi = lo + alpha < nq ? lo + alpha : nq;
        return e >= lo && e < hi;
    }
};
inline RowMap rowmap(int per, int nq, int L) {
    RowMap m;
    m.per = per;
    m.nq = nq;
    m.L = L;
    return m;
}

struct NttTables {
    const u64 *tw, *twp;    // [P][N] psi^brv(i) and Shoup companions
    const u64 *itw, *itwp;  // [P][N] psi^-brv(i)
    // [P][N] pairs of doubles {w, fl(w/q)} for primes below 2^40 (else 0)
    const ulonglong2 *twx, *itwx;
    // [P][N] w as a double for primes below 2^40 (block pass of the 2^16
    // NTT; its fl(w/q) is formed in the kernel)
    const double *tws, *itws;
    int logN;
};

void upload_prime_consts(const PrimeConst *pc, int n);

// ---- launch accounting ------------------------------------------------------
enum KernelClass {
    KC_NTT_FWD, KC_NTT_INV, KC_MODUP_BCONV, KC_MODDOWN_BCONV, KC_MODDOWN_COMBINE, KC_KEYMULT,
    KC_BSGS_MAC, KC_RESCALE, KC_ELEMENTWISE, KC_AUTOMORPHISM, KC_SAMPLE, KC_BSGS_MMA, KC_COUNT
};
struct ProfStats {
    double ms[KC_COUNT] = {};
    double bytes[KC_COUNT] = {};      // algorithmic bytes
    double work[KC_COUNT] = {};       // modular products (NTT: butterflies)
    unsigned long long launches[KC_COUNT] = {};
};
void prof_enable(bool on);             // resets the statistics
void prof_collect(ProfStats *out);     // waits for the recorded events
const char *kclass_name(int c);
unsigned long long launch_count();     // kernels launched since load

// ---- NTT -----------------------------------------------------------------
void ntt_forward(u64 *data, int nrows, RowMap map, const NttTables &t, cudaStream_t s);
void ntt_inverse(u64 *data, int nrows, RowMap map, const NttTables &t, cudaStream_t s);
// out-of-place inverse: dst rows (contiguous) from source items of per_item
// rows at src_stride
void ntt_inverse_from(u64 *dst, const u64 *src, size_t src_stride, int per_item, int nrows, RowMap map,
                      const NttTables &t, cudaStream_t s);

// ---- elementwise ---------------------------------------------------------
// out = a op b on nrows rows (rows map to primes with `map`)
void ew_add(u64 *out, const u64 *a, const u64 *b, int nrows, RowMap map, int logN, cudaStream_t s);
void ew_sub(u64 *out, const u64 *a, const u64 *b, int nrows, RowMap map, int logN, cudaStream_t s);
void ew_neg(u64 *out, const u64 *a, int nrows, RowMap map, int logN, cudaStream_t s);
// out = a mod q(row) for any 64-bit a (sums of residues from several ranks)
void ew_reduce_rows(u64 *out, const u64 *a, int nrows, RowMap map, int logN, cudaStream_t s);
// out[pl][i] = a[pl][i] * b[i]   (b broadcast over npoly blocks of nq rows)
void ew_mul_bcast(u64 *out, const u64 *a, const u64 *b, int npoly, int nq, int b_rows_stride_nq,
                  int logN, cudaStream_t s);
// out[r] = a[r] * c[prime(r)] (+ add[prime(r)] if add != null), constants per prime with Shoup
// one word per prime (and its Shoup companion), passed by value
struct ConstWords {
    u64 v[HB_MAX_PRIMES];
    u64 vp[HB_MAX_PRIMES];
};
void ew_mul_const(u64 *out, const u64 *a, const ConstWords &cw, int nrows, RowMap map, int logN, cudaStream_t s);
void ew_add_const(u64 *out, const u64 *a, const ConstWords &cw, int nrows, RowMap map, int logN, cudaStream_t s);
// ct x ct tensor: out[0]=a0b0, out[1]=a0b1+a1b0, out[2]=a1b1 (nq rows each)
void ew_tensor(u64 *out, const u64 *a, const u64 *b, int nq, int logN, cudaStream_t s);
// out = c0 + c1 * sk (nq rows)
void ew_decrypt(u64 *out, const u64 *ct, const u64 *sk, int nq, int logN, cudaStream_t s);
// automorphism: out[r][t] = in[r][tau_g(t)]
void ew_automorphism(u64 *out, const u64 *in, int nrows, u64 galois, int logN, cudaStream_t s);

#define HB_MAC_MAX 64
struct MacArgs {
    const u64 *ct[HB_MAC_MAX];
    const u64 *pt[HB_MAC_MAX];
    int n;
};
// out[pl][i] = sum_t ct_t[pl][i] * pt_t[i]
void ew_mac(u64 *out, const MacArgs &args, int npoly, int nq, int logN, cudaStream_t s);

// ---- polynomial evaluation -------------------------------------------------------
// nb degree-1 products out[b] = a[b] (x) b[b] ([nb][3][nq][N]); operand items
// sit at strides as / bs and hold anq / bnq rows per polynomial (>= nq)
void ew_tensor_batch(u64 *out, const u64 *a, const u64 *b, int nq, int anq, int bnq, int nb, size_t as, size_t bs,
                     int logN, cudaStream_t s);
#define HB_LC_MAX 48
struct LinCombArgs {
    const u64 *x[HB_LC_MAX];  // operand t: nb ciphertexts, item stride xs[t]
    size_t xs[HB_LC_MAX];
    int nq[HB_LC_MAX];        // rows per polynomial of operand t (>= the output's)
    int n;
    const u64 *coef;          // [n][nq] residues below q_i
    const u64 *k0;            // [nq] residues added to polynomial 0, or null
};
// out[b][pl][i] = sum_t coef[t][i] * x_t[b][pl][i] (+ k0[i] for pl = 0), the
// output's nq rows of each operand, nb degree-1 ciphertexts at out_stride
void ew_lincomb(u64 *out, const LinCombArgs &a, int nq, int nb, size_t out_stride, int logN, cudaStream_t s);

// ---- sampling (counter-based; see hb_kernels.cu) ---------------------------
void sample_uniform(u64 *out, int nrows, const int *row_prime_host_unused, RowMap map, u64 seed, u64 domain,
                    u64 idx_base, u64 idx_row_stride, int logN, cudaStream_t s);
// centred-binomial error, the same integer written modulo every row's prime
void sample_cbd(u64 *out, int nrows, RowMap map, u64 seed, u64 domain, u64 idx_base, int logN,
                cudaStream_t s);

// ---- key generation / encryption combines ------------------------------------
// b = e - a*s (+ pmod[p] * target if addmask row), rows in [0, P)
void swk_combine(u64 *b, const u64 *a, const u64 *e, const u64 *sk, const u64 *target, const u64 *pmod,
                 int nrows, int digit_lo, int digit_hi, int logN, cudaStream_t s);
// c0 = e - a*s + m over nq rows (m may be null)
void enc_combine(u64 *c0, const u64 *a, const u64 *e, const u64 *sk, const u64 *m, int nq, int logN,
                 cudaStream_t s);

// ---- basis conversion --------------------------------------------------------
// ModUp basis conversion for digits [0, beta): X holds the coefficient form
// of the nq input limbs, c1ntt their NTT form.  For every digit j and
// extended row e outside the digit: D[j][e] = sum_m (X_m * qhinv_m mod q_m)
// * qhat_m mod t_e (coefficient form, NTT'd afterwards); rows of the digit
// itself are copied from c1ntt.  The lift is centred: a term y_m above
// q_m/2 stands for y_m - q_m, which adds -Q_j (keeps the digit zero-mean).
// tab: per-level tables in device memory.
struct ModUpTab {
    const u64 *qhinv;   // [beta][alpha]            (and Shoup companions in qhinvp)
    const u64 *qhinvp;
    const u64 *qhat;    // [beta][alpha][ne]        qhat_m mod t_e
    const u64 *qjneg;   // [beta][ne]               t_e - (Q_j mod t_e)
    const u64 *qhat_s;  // qhat in split-30 packed form
    const u64 *qjneg_s; // qjneg in split-30 packed form
    const double2 *qhat_d;  // q-row targets: qhat as {t, fl(t / q_e)} (FP64 modular products)
    const double *qjneg_d;  // q-row targets: qjneg as a double
    int split;          // split products: 1 every main prime below 2^40, 2 every prime below 2^60
};
void modup_bconv(u64 *D, const u64 *X, const u64 *c1ntt, int nq, int K, int L, int alpha, int beta,
                 const ModUpTab &tab, int logN, int nbatch, size_t in_stride, size_t out_stride, size_t c1_stride,
                 cudaStream_t s);

struct ModDownTab {
    const u64 *phinv;   // [K] (P/p_k)^-1 mod p_k, with Shoup
    const u64 *phinvp;
    const u64 *phat;    // [K][nq]  (P/p_k) mod q_i
    const u64 *pinv;    // [nq] P^-1 mod q_i, with Shoup
    const u64 *pinvp;
    const u64 *pneg;    // [nq] q_i - (P mod q_i)
    const u64 *phat_s;  // phat in split-30 packed form
    const u64 *pneg_s;  // pneg in split-30 packed form
    int split;          // split-30 products (nonzero: every prime in the split's range)
};
// Z[i] = sum_k (Y_k * phinv_k mod p_k) * phat_k mod q_i  (coefficient form),
// with the same centred lift as ModUp.
void moddown_bconv(u64 *Z, const u64 *Y, int nq, int K, int L, const ModDownTab &tab, int logN, int nbatch,
                   size_t in_stride, size_t out_stride, cudaStream_t s);
// out[i] = (x[i] - Z[i]) * pinv_i (+ addend[i][tau_g(n)] if addend)
// (+ add2[i] if add2: an unrotated addend, the hybrid fold's c + rot(c))
void moddown_combine(u64 *out, const u64 *x, const u64 *Z, int nq, const ModDownTab &tab, const u64 *addend,
                     u64 add_galois, int logN, int nbatch, size_t x_stride, size_t z_stride,
                     size_t out_stride, size_t add_stride, cudaStream_t s, const u64 *add2 = nullptr,
                     size_t add2_stride = 0);

// ---- rescale ---------------------------------------------------------------
// prep: W[pl][i] = (h mod q_i) - ((R[pl] + h) mod q_l mod q_i), R = INTT of last limb (coef)
void rescale_prep(u64 *W, const u64 *R, int npoly, int nq_out, u64 ql, int logN, int nbatch,
                  size_t r_stride, size_t w_stride, cudaStream_t s);
// out[pl][i] = (c[pl][i] + W[pl][i]) * qlinv_i
void rescale_combine(u64 *out, const u64 *c, const u64 *W, int npoly, int nq_in, const u64 *qlinv,
                     const u64 *qlinvp, int logN, int nbatch, size_t c_stride, size_t w_stride,
                     size_t out_stride, cudaStream_t s);

// ---- key switching -------------------------------------------------------------
// acc[pl][e][n] (+)= sum_{j<beta} D[j][e][tau(n)] * key[j][pl][prime(e)][n]
//                 (+ addb[e][tau(n)] on pl = 0 when addb != null)
// key layout [dnum][2][P][N].  nbatch ciphertexts: D, acc, addb advance by
// their strides, key shared.
void keymult(u64 *acc, const u64 *D, const u64 *key, u64 galois, int nq, int K, int L, int beta, int keyP,
             const u64 *addb, bool accumulate, int logN, int nbatch, size_t d_stride, size_t acc_stride,
             size_t add_stride, cudaStream_t s);
// 2..HB_MAX_GIANTS giant steps of four digits each in one pass (every
// giant with its digits, key, Galois element and unrotated addend)
#define HB_MAX_GIANTS 4
void keymult_group(u64 *acc, int ngiants, const u64 *const *D, const u64 *const *keys, const u64 *galois,
                   const u64 *const *addb, int nq, int K, int L, int beta, int keyP, bool accumulate, int logN,
                   int nbatch, size_t d_stride, size_t acc_stride, size_t add_stride, cudaStream_t s);

// ---- fused double-hoisted baby steps + plaintext MAC --------------------------
#define HB_MAX_BETA 8  // key-switching digits handled by the fused kernels
#define HB_GCH 16   // giant slots per chunk (one warp each)
#define HB_BCH 32   // babies per chunk (plaintexts held in registers)
#define HB_BT 16    // coefficients per thread block tile
struct BabyDesc {
    u64 galois;        // 1 for the identity baby (b = 0)
    const u64 *key;    // null for b = 0
    const u64 *pt[HB_GCH];  // plaintext (ext basis) of (giant slot, this baby) or null
};
struct BsgsChunk {
    const BabyDesc *babies;  // device array
    int nbabies;
    int gbase;               // first output giant slot of this chunk
    int gcount;              // giant slots in this chunk (<= HB_GCH)
    int nkeys;               // babies with a key (b != 0), for accounting
    int npts;                // plaintexts referenced by the chunk, for accounting
    int accumulate;          // add into inner (later baby chunks of the same giant slots)
    const uint8_t *ptp;      // plaintext byte planes of the q rows (tensor-core MAC), or null
};
// inner[g][pl][e][n] for g in [gbase, gbase+gcount): sum over babies of
// pt(g, b) * R_b, R_b = baby rotation of the input kept in the PQ basis:
// R_b.b = P*c0[tau] + sum_j D_j[tau] key.b,  R_b.a = sum_j D_j[tau] key.a.
void bsgs_baby_mac(u64 *inner, const u64 *ct, const u64 *D, const BsgsChunk &ch, int nq, int K, int L,
                   int beta, int keyP, int pt_nq, const u64 *pmod_q, int logN, int nbatch, size_t ct_stride,
                   size_t d_stride, size_t inner_stride, cudaStream_t s);

// ---- one-pass table x ciphertext-vector products (IVE lookup) -----------------
struct MatMulArgs {
    u64 *const *out;          // device array: rows output ciphertexts [2][nq][N]
    const u64 *const *x;      // device array: 2 * cols pointers (poly 0, poly 1 of each input)
    const double *tab;        // constants [nq][rows][cols] (exact doubles), or null
    const u64 *const *pts;    // plaintext table [rows][cols] of q-row pointers, or null
    int rows, cols, nq, logN;
    int r0;                   // first row of the launch (set by the launcher)
};
// out_r = sum_k T[r][k] * x_k over the q rows of every limb; primes below 2^40
void table_matmul(const MatMulArgs &args, bool pt, cudaStream_t s);

// ---- the same MAC on the tensor cores (q rows; hb_bsgs_tc.cuh) ----------------
// Usable when every q row prime is below 2^37, the chunk has at most 32
// babies and 16 giant slots, and beta is 1..4.
bool bsgs_mma_supported(int nq, int beta);
// bytes of the plaintext byte planes of one chunk (q rows nq)
size_t bsgs_mma_planes_bytes(int nq, int logN);
// ch.ptp <- the chunk's plaintexts as byte planes (one launch)
void bsgs_mma_planes(uint8_t *ptp, const BsgsChunk &ch, int nq, int logN, cudaStream_t s);
// [nq][9] table 2^(8s) mod q_e for the epilogue (host values)
void bsgs_mma_class_consts(u64 *out, const u64 *primes, int nq);
// inner[g][pl][e][n] for the q rows e < nq, over nbatch ciphertexts in
// passes of 32; the special rows are left to bsgs_baby_mac_special.
// err: device word receiving HB_TC_ERR_* bits if a pipeline wait ran out.
void bsgs_baby_mma(u64 *inner, const u64 *ct, const u64 *D, const BsgsChunk &ch, const u64 *cls, int nq, int K,
                   int L, int beta, int keyP, const u64 *pmod_q, int logN, int nbatch, size_t ct_stride,
                   size_t d_stride, size_t inner_stride, int *err, cudaStream_t s);
// the CUDA-core MAC on the special-prime rows only
void bsgs_baby_mac_special(u64 *inner, const u64 *ct, const u64 *D, const BsgsChunk &ch, int nq, int K, int L,
                           int beta, int keyP, int pt_nq, const u64 *pmod_q, int logN, int nbatch,
                           size_t ct_stride, size_t d_stride, size_t inner_stride, cudaStream_t s);

// copy rows with optional automorphism (used to place P*c parts etc.)
void copy_rows(u64 *dst, const u64 *src, size_t nwords, cudaStream_t s);

// ---- batched copies (one launch per batch; words, strides and pointers are
// whole limbs, so 16-byte aligned) ------------------------------------------------
// dst[b * dstride + i] = src[b * sstride + i] for i < words, b < nb
void copy_strided(u64 *dst, size_t dstride, const u64 *src, size_t sstride, size_t words, int nb, cudaStream_t s);
#define HB_PTR_BATCH 128
struct PtrBatch {
    const u64 *p[HB_PTR_BATCH];
};
struct PtrBatchW {
    u64 *p[HB_PTR_BATCH];
};
// dst[b][j * words + i] = seg_j.p[b][i] for the nseg (1 or 2) segments of item b
void gather_items(u64 *dst, const PtrBatch &seg0, const PtrBatch &seg1, int nseg, size_t words, int nb,
                  cudaStream_t s);
// dst.p[b][i] = src[b * words + i]
void scatter_items(const PtrBatchW &dst, const u64 *src, size_t words, int nb, cudaStream_t s);

// ---- device CKKS encoding ------------------------------------------------------
// perm[j]: bit-reversed position of slot j in the length-N/2 transform;
// tw[k] = exp(-2 pi i k / (N/2)), k < N/4
struct EncTables {
    const int *perm;
    const double2 *tw;
    int logN;
};
void enc_tables(int *perm, double2 *tw, int logN, cudaStream_t s);
// decoding: Garner constants of the first n limbs (mmod[i][k] = q_0 .. q_{k-1}
// mod q_i, minv[i] its inverse at k = i); out <- the slots (interleaved re, im
// when cplx) of the plaintext whose first n limbs (coefficient form, after the
// inverse NTT) are at limbs; coef (N doubles) and z (N/2 complex) are scratch
#define HB_DEC_MAX 4
struct DecCrt {
    int n;
    u64 mmod[HB_DEC_MAX * HB_DEC_MAX];
    u64 minv[HB_DEC_MAX];
};
void decode_slots(double *out, const u64 *limbs, const DecCrt &c, double scale, int cplx, double *coef, double2 *z,
                  const EncTables &t, cudaStream_t s);
// z[v] <- the nvals slot values of vector v (interleaved re, im when cplx, else
// real), zero in the other slots, in the transform's input order
void enc_scatter(double2 *z, const double *vals, int nvals, int cplx, int count, const EncTables &t, cudaStream_t s);
// in-place unnormalised inverse DFT of every vector
void enc_ifft(double2 *z, int count, const EncTables &t, cudaStream_t s);
// coefficients of vector v as residues on `rows` rows of `map` into dst.p[v]
// (coefficient order; |scale * value| below 2^62)
void enc_round(const PtrBatchW &dst, const double2 *z, int rows, RowMap map, double scale, int count,
               const EncTables &t, cudaStream_t s);
// bootstrapping's ModRaise: the coefficient-form rows co[2][N] (modulo q_0),
// lifted centred, as residues of the first nq main primes into out[2][nq][N]
void mod_raise_rows(u64 *out, const u64 *co, int nq, int logN, cudaStream_t s);
// out = i * in slot-wise (multiplication by X^(N/2)): nrows rows, prime of
// row r is r % nq, iu = [P][4] {w, w', q - w, (q - w)'} (w = psi^(N/2))
void ew_mul_iunit(u64 *out, const u64 *in, int nrows, int nq, const u64 *iu, int logN, cudaStream_t s);
// lane split of nb packed ciphertexts p and their conjugates c (both
// contiguous [nb][2][nq][N]): ev.p[b] = p + c, od.p[b] = i (c - p)
void lane_split(const PtrBatchW &ev, const PtrBatchW &od, const u64 *pk, const u64 *cj, int nq, int nb, const u64 *iu,
                int logN, cudaStream_t s);

}  // namespace hb
