// hb_context.cu -- scheme state, object registries, the CKKS operations
// built from the kernels in hb_kernels.cu, and the extern "C" boundary
// declared in include/helrm_b200.h.
//
// Ownership follows the reference backends: the library owns every
// ciphertext, plaintext and transform; callers hold int handles
// (orion/backend/cheddar/ext/cheddar_pybind.cu:73-236).  All device work
// goes to one non-blocking stream; memory comes from CUDA's stream-ordered
// pool (cudaMallocAsync), which keeps freed blocks cached for reuse.
#include <cuda_profiler_api.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "../../include/helrm_b200.h"
#include "hb_host.hpp"
#include "hb_kernels.cuh"

// Giant steps of the double-hoisted LT per key-multiplication launch (four
// digits; at most HB_MAX_GIANTS): the PQ accumulator is read and written
// once per group.  Three measured fastest on B200 (two: 28.0 ms, three:
// 26.1 ms, four: 27.7 ms of key multiplication per cfg2 step).
#ifndef HB_LT_GIANT_GROUP
#define HB_LT_GIANT_GROUP 3
#endif
static_assert(HB_LT_GIANT_GROUP >= 1 && HB_LT_GIANT_GROUP <= HB_MAX_GIANTS, "giant group size");
// Ciphertexts per launch of the CUDA-core baby-step MAC (HELRM_B200_MAC_CHUNK
// overrides).
#ifndef HB_MAC_CT_CHUNK
#define HB_MAC_CT_CHUNK 64
#endif

namespace hb {

struct HbError : std::runtime_error {
    int code;
    HbError(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};
#define HB_THROW(code, msg) throw HbError(code, msg)

static void cuda_check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) {
        if (e == cudaErrorMemoryAllocation) HB_THROW(HB_ENOMEM, std::string(what) + ": out of device memory");
        HB_THROW(HB_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
    }
}

enum : u64 {
    DOM_SK_POS = 1, DOM_SK_SIGN = 2, DOM_ENC_A = 3, DOM_ENC_E = 4,
    DOM_SWK_A = 5, DOM_SWK_E = 6, DOM_KEYSEED = 7, DOM_PK_A = 8, DOM_PK_E = 9
};

static inline u64 hmix(u64 z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static inline u64 hrand64(u64 seed, u64 dom, u64 idx) { return hmix(hmix(seed ^ hmix(dom)) ^ idx); }

struct Ct {
    u64 *d = nullptr;
    int nq = 0;
    int npoly = 2;
    double scale = 1.0;
    int slots = 0;
    bool xfer = false;  // an asynchronous download may still read d: free behind it
};
struct Pt {
    u64 *d = nullptr;
    int nq = 0;      // q rows
    bool ext = false;  // K special-prime rows follow
    double scale = 1.0;
    int slots = 0;
};

struct LevelTabs {
    // device blob; pointers into it
    u64 *blob = nullptr;
    ModUpTab mu{};
    ModDownTab md{};
    const u64 *qlinv = nullptr, *qlinvp = nullptr;
    int beta = 0;
};

struct LinTrans {
    int level = 0;
    double scale = 0.0;                           // plaintext scale of the diagonals
    int bs = 1;
    bool use_bsgs = false;
    std::vector<int> ks;
    std::map<int, Pt> pts;                        // k -> extended plaintext
    std::map<int, std::vector<std::pair<int, int>>> groups;  // g -> (b, k)
    // device plans, rebuilt when the rotation-key set changes
    int plan_keygen = -1;
    int plan_nq = -1;
    std::vector<BabyDesc *> plan_dev;
    std::vector<BsgsChunk> plan_chunks;
    std::vector<int> giant_of_slot;   // slot -> g
};

// ---- polynomial evaluation plans --------------------------------------------
// EvaluatePolynomial (orion/backend/python/poly_evaluator.py:25-35, bound by
// orion/backend/cheddar/bindings.py:1102-1116 to the native EvalPoly of
// cheddar_pybind.cu:2207-2262) evaluates sum_j c_j T_j(x) (Chebyshev basis)
// or sum_j c_j x^j with ceil(log2(d+1)) levels, the depth orion/nn/
// activation.py:22-28,101-110 places the layers with, and returns exactly the
// requested output scale.  The evaluation is the baby-step giant-step
// recursion (Paterson-Stockmeyer in the Chebyshev basis, as published by
// Bossuat, Mouchet, Troncoso-Pastoriza and Hubaux, Eurocrypt 2021):
//   p = q * T_{2^k} + r,  2^k <= deg p < 2^(k+1),
// with q evaluated one level higher at scale S q_{L+1} / s(T_{2^k}), the
// product and the remainder's leaf sum  sum_i round(r_i S q_{L+1} / s_i) T_i
// + round(r_0 S q_{L+1})  added before one rescale, so every node lands on
// its target scale exactly.  A node is a leaf when all its powers are in the
// basis (T_1..T_bs and the powers of two) at a level above its target.  In
// the basis, T_{a+b} = 2 T_a T_b - T_{a-b} is formed before its rescale as
// 2 T_a T_b - K T_{a-b}, K = round(s_a s_b / s_{a-b}) (an integer multiple:
// no level, a relative scale error below 2^-36), and T_{2a} = 2 T_a^2 - 1.
// The host builds the whole evaluation as a plan of four device operations
// (product with relinearization, linear combination, rescale, add), picks
// the baby-step count bs in {2, 4, .., 32} with the fewest products, and
// replays the plan over a batch of ciphertexts.
enum { PO_MUL, PO_LIN, PO_RESCALE, PO_ADD };
struct PolyOp {
    int kind = 0;
    int out = 0, a = -1, b = -1;  // value ids
    int t0 = 0, nt = 0;           // PO_LIN: operand value ids terms[t0 .. t0 + nt)
    size_t coef = 0;              // PO_LIN: offset of the [nt][nq] residues in consts
    long k0 = -1;                 // PO_LIN: offset of the [nq] constant's residues, or -1
};
struct PolyPlan {
    int bs = 0, depth = 0, products = 0, rescales = 0;
    double target = 0;
    std::vector<PolyOp> ops;
    std::vector<int> terms;
    std::vector<int> vnq;        // rows per polynomial of each value (value 0 = the input)
    std::vector<double> vscale;
    std::vector<int> last_use;   // index of the last op reading each value
    std::vector<u64> consts;     // host residues
    u64 *d_consts = nullptr;
    int out = 0;
};

static int poly_ceil_log2(long v) {
    int k = 0;
    while ((1L << k) < v) k++;
    return k;
}
static long poly_floor_pow2(long v) {
    long p = 1;
    while (p * 2 <= v) p *= 2;
    return p;
}
static int poly_degree(const std::vector<double> &c) {
    int d = (int)c.size() - 1;
    while (d > 0 && c[d] == 0.0) d--;
    return d < 0 ? 0 : d;
}

class PolyPlanner {
public:
    PolyPlanner(const std::vector<u64> &primes, bool cheb, int nq0, double s1, int bs)
        : primes_(primes), cheb_(cheb), nq0_(nq0), bs_(bs) {
        p.bs = bs;
        value(nq0, s1);
        tv_[1] = 0;
    }
    // plan the evaluation of c to `levels` levels below the input at scale S
    PolyPlan build(const std::vector<double> &c, int levels, double S) {
        const int L = nq0_ - 1 - levels;
        if (L < 0) HB_THROW(HB_ESTATE, "EvaluatePolynomial: not enough levels for the polynomial's degree.");
        p.depth = levels;
        p.target = S;
        p.out = eval(c, L, S);
        p.last_use.assign(p.vnq.size(), -1);
        for (size_t i = 0; i < p.ops.size(); i++) {
            const PolyOp &o = p.ops[i];
            if (o.a >= 0) p.last_use[o.a] = (int)i;
            if (o.b >= 0) p.last_use[o.b] = (int)i;
            for (int t = 0; t < o.nt; t++) p.last_use[p.terms[o.t0 + t]] = (int)i;
        }
        return std::move(p);
    }

private:
    typedef std::vector<std::pair<int, double>> Terms;
    const std::vector<u64> &primes_;
    bool cheb_;
    int nq0_, bs_;
    PolyPlan p;
    std::map<long, int> tv_;  // power index -> value id

    int value(int nq, double scale) {
        p.vnq.push_back(nq);
        p.vscale.push_back(scale);
        return (int)p.vnq.size() - 1;
    }
    double q(int nq) const { return (double)primes_[nq - 1]; }
    // round half away from zero, then one residue per prime of the first nq
    void residues(double v, int nq) {
        const double r = std::round(v);
        if (!(std::fabs(r) < 1.0e38)) HB_THROW(HB_EINVAL, "EvaluatePolynomial: a coefficient times its scale overflows");
        const hi128 x = (hi128)r;
        for (int i = 0; i < nq; i++) {
            const u64 m = (u64)((hu128)(x < 0 ? -x : x) % primes_[i]);
            p.consts.push_back(x < 0 && m ? primes_[i] - m : m);
        }
    }
    int mul(int a, int b) {
        const int nq = std::min(p.vnq[a], p.vnq[b]);
        const int v = value(nq, p.vscale[a] * p.vscale[b]);
        PolyOp o;
        o.kind = PO_MUL, o.out = v, o.a = a, o.b = b;
        p.ops.push_back(o);
        p.products++;
        return v;
    }
    int lin(int nq, double scale, const Terms &t, bool has_k0, double k0) {
        if ((int)t.size() > HB_LC_MAX) HB_THROW(HB_ESTATE, "EvaluatePolynomial: leaf wider than the combination kernel");
        const int v = value(nq, scale);
        PolyOp o;
        o.kind = PO_LIN, o.out = v, o.t0 = (int)p.terms.size(), o.nt = (int)t.size(), o.coef = p.consts.size();
        for (auto &x : t) {
            if (p.vnq[x.first] < nq) HB_THROW(HB_ESTATE, "EvaluatePolynomial: operand below the node's level");
            p.terms.push_back(x.first);
            residues(x.second, nq);
        }
        if (has_k0) {
            o.k0 = (long)p.consts.size();
            residues(k0, nq);
        }
        p.ops.push_back(o);
        return v;
    }
    int rescale(int a, double scale) {
        if (p.vnq[a] < 2) HB_THROW(HB_ESTATE, "EvaluatePolynomial: rescale below level 0");
        const int v = value(p.vnq[a] - 1, scale);
        PolyOp o;
        o.kind = PO_RESCALE, o.out = v, o.a = a;
        p.ops.push_back(o);
        p.rescales++;
        return v;
    }
    int add(int a, int b) {
        if (p.vnq[a] != p.vnq[b]) HB_THROW(HB_ESTATE, "EvaluatePolynomial: adding nodes of different levels");
        const int v = value(p.vnq[a], p.vscale[a]);
        PolyOp o;
        o.kind = PO_ADD, o.out = v, o.a = a, o.b = b;
        p.ops.push_back(o);
        return v;
    }
    bool pow2(long i) const { return (i & (i - 1)) == 0; }
    int nq_of_power(long i) const { return nq0_ - poly_ceil_log2(i); }
    // T_i (or x^i), its rows nq0 - ceil(log2 i)
    int power(long i) {
        auto it = tv_.find(i);
        if (it != tv_.end()) return it->second;
        int v;
        if (!cheb_) {
            const long a = pow2(i) ? i / 2 : poly_floor_pow2(i), b = i - a;
            const int va = power(a), vb = power(b);
            const int P = mul(va, vb);
            v = rescale(P, p.vscale[P] / q(p.vnq[P]));
        } else if (pow2(i)) {
            const int va = power(i / 2);
            const int P = mul(va, va);
            const double sp = p.vscale[P];
            const int Lv = lin(p.vnq[P], sp, Terms{{P, 2.0}}, true, -sp);
            v = rescale(Lv, sp / q(p.vnq[P]));
        } else {
            const long a = poly_floor_pow2(i), b = i - a, c = a - b;
            const int va = power(a), vb = power(b), vc = power(c);
            const int P = mul(va, vb);
            const double sp = p.vscale[P];
            const double K = std::round(sp / p.vscale[vc]);
            const int Lv = lin(p.vnq[P], sp, Terms{{P, 2.0}, {vc, -K}}, false, 0.0);
            v = rescale(Lv, sp / q(p.vnq[P]));
        }
        tv_[i] = v;
        return v;
    }
    bool leafable(const std::vector<double> &c, int L) const {
        for (size_t i = 1; i < c.size(); i++) {
            if (c[i] == 0.0) continue;
            if (!((long)i <= bs_ || pow2((long)i)) || nq_of_power((long)i) < L + 2) return false;
        }
        return true;
    }
    double leaf_terms(const std::vector<double> &c, double Sp, Terms &t) {
        for (size_t i = 1; i < c.size(); i++) {
            if (c[i] == 0.0) continue;
            const int v = power((long)i);
            t.push_back({v, (c[i] * Sp) / p.vscale[v]});
        }
        return c[0] * Sp;
    }
    // a ciphertext of c at level L (L + 1 rows) and scale exactly S
    int eval(const std::vector<double> &c0, int L, double S) {
        const int d = poly_degree(c0);
        const std::vector<double> c(c0.begin(), c0.begin() + d + 1);
        const double Sp = S * q(L + 2);
        if (leafable(c, L)) {
            Terms t;
            const double k0 = leaf_terms(c, Sp, t);
            if (t.empty()) t.push_back({power(1), 0.0});
            return rescale(lin(L + 2, Sp, t, true, k0), S);
        }
        const long n2 = poly_floor_pow2(d);
        std::vector<double> qv((size_t)(d - n2 + 1)), rv(c.begin(), c.begin() + n2);
        if (cheb_) {
            qv[0] = c[n2];
            for (long i = 1; i <= d - n2; i++) {
                qv[i] = 2.0 * c[n2 + i];
                rv[n2 - i] -= c[n2 + i];
            }
        } else {
            for (long i = 0; i <= d - n2; i++) qv[i] = c[n2 + i];
        }
        const int G = power(n2);
        if (p.vnq[G] < L + 2) HB_THROW(HB_ESTATE, "EvaluatePolynomial: giant step below the node's level");
        Terms t;
        const bool qconst = poly_degree(qv) == 0;
        if (qconst)
            t.push_back({G, (qv[0] * Sp) / p.vscale[G]});
        else
            t.push_back({mul(eval(qv, L + 1, Sp / p.vscale[G]), G), 1.0});
        if (leafable(rv, L)) {
            const double k0 = leaf_terms(rv, Sp, t);
            return rescale(lin(L + 2, Sp, t, true, k0), S);
        }
        const int R = eval(rv, L, S);
        const int v = qconst ? lin(L + 2, Sp, t, false, 0.0) : t[0].first;
        return add(rescale(v, S), R);
    }
};

// the plan with the fewest products (then rescales) over bs = 2 .. 32
static PolyPlan plan_polynomial(const std::vector<u64> &primes, bool cheb, int nq0, double s1,
                                const std::vector<double> &c, double S) {
    if (c.size() < 3) HB_THROW(HB_EINVAL, "EvaluatePolynomial: the native evaluation needs degree >= 2");
    const int levels = poly_ceil_log2((long)c.size());
    PolyPlan best;
    bool have = false;
    for (int bs = 2; bs <= 32 && bs <= (1 << levels); bs *= 2) {
        PolyPlan cand = PolyPlanner(primes, cheb, nq0, s1, bs).build(c, levels, S);
        if (!have || cand.products < best.products ||
            (cand.products == best.products && cand.rescales < best.rescales)) {
            best = std::move(cand);
            have = true;
        }
    }
    return best;
}

// ---- fixed scratch of the no-allocation rescale -----------------------------
// Some callers must not allocate device memory at all: a host runtime that
// reserves the whole HBM budget up front through its own allocator (an
// allocation behind its back can fail or push its pool out of memory), and
// serving loops where the first request of a new batch size would otherwise
// grow the stream-ordered pool with a blocking cudaMalloc in the middle of a
// latency-critical step.  For them helrm_kernel_rescale_noalloc takes its
// temporaries from this fixed array, part of the library's device image.
// Every word the call reads from it is written earlier in the same call, so
// nothing in it has to start at zero and it is never cleared.
static __device__ __align__(256) u64 g_rescale_scratch[HELRM_RESCALE_SCRATCH_WORDS];

// The array's device address on the current device.  In host code the
// symbol is only a host-side stand-in, so kernels get this address instead.
// Called with the scheme's device current when the scheme is created (the
// lookup loads the library's device image on that device), so the address
// always belongs to the live context.
static u64 *lookup_rescale_scratch() {
    void *p = nullptr;
    cuda_check(cudaGetSymbolAddress(&p, g_rescale_scratch), "cudaGetSymbolAddress(rescale scratch)");
    if (!p) HB_THROW(HB_ECUDA, "cudaGetSymbolAddress(rescale scratch) returned null");
    return (u64 *)p;
}

class Context {
public:
    int device = 0;
    int logN = 0, N = 0, L = 0, K = 0, P = 0, alpha = 1, dnum = 1, logscale = 0, h = 0, slots = 0;
    u64 seed = 0;
    double default_scale = 1.0;
    std::vector<u64> primes;
    cudaStream_t stream = nullptr;
    NttTables ntt{};
    u64 *d_tables = nullptr;
    u64 *d_pmod = nullptr;     // P mod q_p, [P]
    u64 *d_cls8 = nullptr;     // [L][9] 2^(8s) mod q_i (tensor-core MAC epilogue)
    u64 *d_iunit = nullptr;    // [P][4] w, w', q - w, (q - w)': X^(N/2) in the NTT order (w = psi^(N/2))
    int *d_enc_perm = nullptr;     // device encoding: slot -> transform position
    double2 *d_enc_tw = nullptr;   // device encoding: exp(-2 pi i k / (N/2))
    int *d_tc_err = nullptr;   // error bits of the tensor-core MAC's bounded waits
    bool use_tc = false;       // tensor-core baby-step MAC where supported (HELRM_B200_MAC=tc)
    std::vector<LevelTabs> lv; // index nq (1..L)
    std::vector<PrimeConst> pcs;
    // keys
    u64 *d_sk = nullptr;
    u64 *d_rlk = nullptr;
    std::map<u64, u64 *> rot_keys;  // galois -> [dnum][2][P][N]
    int keygen_counter = 0;
    // registries
    std::unordered_map<int, Ct> cts;
    std::unordered_map<int, Pt> pts;
    std::unordered_map<int, std::unique_ptr<LinTrans>> lts;
    // broadcast constants (one word per prime) and the IVE lookup's tables
    struct Konst {
        int level = 0;
        double scale = 1.0;
        std::vector<u64> words;  // [level + 1]
    };
    struct Table {
        int rows = 0, cols = 0, level = 0;
        double scale = 1.0;
        bool pt = false;
        double *tab = nullptr;        // constants [nq][rows][cols] (device)
        std::vector<int> pt_ids;      // plaintext table, row-major (kept by id)
    };
    std::unordered_map<int, Konst> konsts;
    std::unordered_map<int, Table> tables;
    // polynomial evaluation plans by basis, input rows and scale, output
    // scale and coefficients (device residues uploaded once per plan)
    std::map<std::string, PolyPlan> poly_plans;
    int next_id = 1;
    u64 enc_counter = 0;
    // memory accounting
    std::unordered_map<void *, size_t> alloc_sizes;
    size_t live = 0, peak = 0, key_bytes = 0;
    u64 n_allocs = 0;  // device-pool allocations made through alloc()/alloc_on()
    // device address of the fixed rescale scratch array on this scheme's
    // device, looked up once when the scheme is created
    u64 *d_rescale_scratch = nullptr;

    size_t limb_bytes() const { return (size_t)N * sizeof(u64); }
    size_t key_words() const { return (size_t)dnum * 2 * P * N; }

    // ---------------------------------------------------------- memory
    u64 *alloc(size_t words) {
        void *p = nullptr;
        if (words == 0) words = 1;
        cuda_check(cudaMallocAsync(&p, words * sizeof(u64), stream), "cudaMallocAsync");
        n_allocs++;
        alloc_sizes[p] = words * sizeof(u64);
        live += words * sizeof(u64);
        peak = std::max(peak, live);
        return (u64 *)p;
    }
    void release(void *p, cudaStream_t on = nullptr) {
        if (!p) return;
        auto it = alloc_sizes.find(p);
        if (it != alloc_sizes.end()) {
            live -= it->second;
            alloc_sizes.erase(it);
        }
        cudaFreeAsync(p, on ? on : stream);
    }
    u64 *alloc_on(size_t words, cudaStream_t s) {
        void *p = nullptr;
        if (words == 0) words = 1;
        cuda_check(cudaMallocAsync(&p, words * sizeof(u64), s), "cudaMallocAsync");
        n_allocs++;
        alloc_sizes[p] = words * sizeof(u64);
        live += words * sizeof(u64);
        peak = std::max(peak, live);
        return (u64 *)p;
    }

    // ---------------------------------------------------------- transfer streams
    // Host <-> device copies of whole ciphertexts run on two more streams, one
    // per direction (PCIe is full duplex), so that they overlap each other and
    // the arithmetic on `stream`; events order the streams.
    cudaStream_t up = nullptr, dn = nullptr;
    cudaEvent_t ev_up = nullptr, ev_dn = nullptr, ev_comp = nullptr;
    void ensure_xfer() {
        if (up) return;
        cuda_check(cudaStreamCreateWithFlags(&up, cudaStreamNonBlocking), "upload stream");
        cuda_check(cudaStreamCreateWithFlags(&dn, cudaStreamNonBlocking), "download stream");
        cuda_check(cudaEventCreateWithFlags(&ev_up, cudaEventDisableTiming), "event");
        cuda_check(cudaEventCreateWithFlags(&ev_dn, cudaEventDisableTiming), "event");
        cuda_check(cudaEventCreateWithFlags(&ev_comp, cudaEventDisableTiming), "event");
    }
    // `on` waits for everything issued on `after` so far
    void wait_for(cudaStream_t on, cudaStream_t after, cudaEvent_t ev) {
        cuda_check(cudaEventRecord(ev, after), "event");
        cuda_check(cudaStreamWaitEvent(on, ev, 0), "wait");
    }
    void sync_xfer() {
        if (up) cuda_check(cudaStreamSynchronize(up), "upload sync");
        if (dn) cuda_check(cudaStreamSynchronize(dn), "download sync");
    }
    // free a ciphertext's memory; behind both the arithmetic and the download
    // stream when a download may be in flight
    void release_ct(Ct &c) {
        if (c.xfer && dn) {
            wait_for(dn, stream, ev_comp);
            release(c.d, dn);
        } else {
            release(c.d);
        }
        c.d = nullptr;
    }
    void zero(u64 *p, size_t words) { cuda_check(cudaMemsetAsync(p, 0, words * 8, stream), "memset"); }
    void d2d(u64 *dst, const u64 *src, size_t words) {
        cuda_check(cudaMemcpyAsync(dst, src, words * 8, cudaMemcpyDeviceToDevice, stream), "d2d");
    }
    void sync() {
        cuda_check(cudaStreamSynchronize(stream), "sync");
        check_tc_error();
    }
    // a tensor-core MAC pipeline wait that ran out leaves its bits in d_tc_err
    void check_tc_error() {
        if (!d_tc_err) return;
        int v = 0;
        cuda_check(cudaMemcpy(&v, d_tc_err, sizeof(int), cudaMemcpyDeviceToHost), "tc error word");
        if (v) {
            cudaMemset(d_tc_err, 0, sizeof(int));
            HB_THROW(HB_ECUDA, "tensor-core MAC: a pipeline wait timed out (bits " + std::to_string(v) +
                                   "); its output is invalid");
        }
    }

    RowMap qmap(int nq) const { return rowmap(nq, nq, L); }
    RowMap extmap(int nq) const { return rowmap(nq + K, nq, L); }
    int beta_of(int nq) const { return (nq + alpha - 1) / alpha; }

    // ---------------------------------------------------------- setup
    void setup(int logn, const std::vector<int> &logq, const std::vector<int> &logp, int lscale, int hw, int dn,
               u64 sd, int dev) {
        if (logn < 10 || logn > 17) HB_THROW(HB_EINVAL, "LogN must be in [10, 17]");
        if (logq.empty() || logp.empty()) HB_THROW(HB_EINVAL, "LogQ and LogP must be non-empty");
        if ((int)(logq.size() + logp.size()) > HB_MAX_PRIMES) HB_THROW(HB_EINVAL, "too many primes");
        if (logp.size() > 8) HB_THROW(HB_EINVAL, "at most 8 special primes");
        for (int b : logq)
            if (b > 60) HB_THROW(HB_EINVAL, "prime sizes above 60 bits are not supported (lazy 128-bit sums)");
        for (int b : logp)
            if (b > 60) HB_THROW(HB_EINVAL, "prime sizes above 60 bits are not supported (lazy 128-bit sums)");
        device = dev;
        cuda_check(cudaSetDevice(dev), "cudaSetDevice");
        logN = logn;
        N = 1 << logn;
        slots = N / 2;
        L = (int)logq.size();
        K = (int)logp.size();
        P = L + K;
        logscale = lscale;
        default_scale = std::ldexp(1.0, lscale);
        h = hw;
        seed = sd;
        std::vector<u64> used;
        primes = gen_primes(logq, logn, used);
        std::vector<u64> aux = gen_primes(logp, logn, used);
        primes.insert(primes.end(), aux.begin(), aux.end());
        // digits: dnum given, or Lattigo's default of |P| primes per digit
        alpha = dn > 0 ? (L + dn - 1) / dn : K;
        if (alpha < 1) alpha = 1;
        if (alpha > 16) HB_THROW(HB_EINVAL, "digits of more than 16 primes are not supported");
        dnum = (L + alpha - 1) / alpha;
        if (dnum > HB_MAX_BETA)
            HB_THROW(HB_EINVAL, "more than " + std::to_string(HB_MAX_BETA) +
                                    " key-switching digits; pass a smaller dnum or more special primes");

        cuda_check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
        d_rescale_scratch = lookup_rescale_scratch();
        cudaMemPool_t pool;
        cuda_check(cudaDeviceGetDefaultMemPool(&pool, dev), "mempool");
        u64 thr = ~0ull;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);

        // per-prime constants
        pcs.resize(P);
        for (int p = 0; p < P; p++) {
            u64 q = primes[p];
            PrimeConst c;
            c.q = q;
            c.r64 = (u64)(((hu128)1 << 64) % q);
            c.r64p = h_shoup(c.r64, q);
            c.onep = (u64)(((hu128)1 << 64) / q);
            c.ninv = h_invm((u64)N, q);
            c.ninvp = h_shoup(c.ninv, q);
            c.c60 = (1ull << 60) % q;
            c.c60p = h_shoup(c.c60, q);
            c.c58 = (1ull << 58) % q;
            c.c58p = h_shoup(c.c58, q);
            c.qinv = 1.0 / (double)q;
            c.c58d = (double)c.c58;
            c.c90 = h_mulm((1ull << 60) % q, (1ull << 30) % q, q);
            c.c60d = (double)c.c60;
            c.c90d = (double)c.c90;
            pcs[p] = c;
        }
        upload_prime_consts(pcs.data(), P);

        // twiddles
        // [4][P][N] u64 twiddles and Shoup companions, then [2][P][N] pairs
        // {w, fl(w/q)} for primes below 2^40 (quotient estimates of the NTT)
        std::vector<u64> tw((size_t)10 * P * N, 0);
        for (int p = 0; p < P; p++) {
            u64 q = primes[p];
            u64 psi = find_psi(q, logN), ipsi = h_invm(psi, q);
            u64 *T = &tw[(size_t)(0 * P + p) * N], *Tp = &tw[(size_t)(1 * P + p) * N];
            u64 *I = &tw[(size_t)(2 * P + p) * N], *Ip = &tw[(size_t)(3 * P + p) * N];
            u64 w = 1, iw = 1;
            for (int i = 0; i < N; i++) {
                unsigned r = h_brv((unsigned)i, logN);
                T[r] = w;
                I[r] = iw;
                w = h_mulm(w, psi, q);
                iw = h_mulm(iw, ipsi, q);
            }
            for (int i = 0; i < N; i++) {
                Tp[i] = h_shoup(T[i], q);
                Ip[i] = h_shoup(I[i], q);
            }
            if (q < (1ull << 40)) {
                u64 *Tx = &tw[(size_t)4 * P * N + (size_t)p * 2 * N];
                u64 *Ix = &tw[(size_t)6 * P * N + (size_t)p * 2 * N];
                for (int i = 0; i < N; i++) {
                    // both operands exact doubles: the quotient is correctly rounded
                    const double tq = (double)T[i] / (double)q, iq = (double)I[i] / (double)q;
                    // pairs of doubles {w, fl(w/q)} (double-precision butterflies)
                    const double td = (double)T[i];
                    std::memcpy(&Tx[2 * i], &td, 8);
                    std::memcpy(&Tx[2 * i + 1], &tq, 8);
                    const double id = (double)I[i];
                    std::memcpy(&Ix[2 * i], &id, 8);
                    std::memcpy(&Ix[2 * i + 1], &iq, 8);
                }
                if (logN == 16) {
                    // single doubles w for the block pass; in the segment of
                    // the 2^15-group stage (16 threads x 8 values) value i of
                    // thread c is stored at 64 (i / 4) + 4 c + (i % 4)
                    double *Ts = reinterpret_cast<double *>(&tw[(size_t)(8 * P + p) * N]);
                    double *Is = reinterpret_cast<double *>(&tw[(size_t)(9 * P + p) * N]);
                    for (int i = 0; i < N; i++) {
                        size_t dst = (size_t)i;
                        if (i >= 32768) {
                            const int b0 = i & ~127, r = i & 127, c = r >> 3, k = r & 7;
                            dst = (size_t)b0 + 64 * (k >> 2) + 4 * c + (k & 3);
                        }
                        Ts[dst] = (double)T[i];
                        Is[dst] = (double)I[i];
                    }
                }
            }
        }
        d_tables = alloc(tw.size());
        cuda_check(cudaMemcpyAsync(d_tables, tw.data(), tw.size() * 8, cudaMemcpyHostToDevice, stream), "tw upload");
        ntt.tw = d_tables;
        ntt.twp = d_tables + (size_t)P * N;
        ntt.itw = d_tables + (size_t)2 * P * N;
        ntt.itwp = d_tables + (size_t)3 * P * N;
        ntt.twx = reinterpret_cast<const ulonglong2 *>(d_tables + (size_t)4 * P * N);
        ntt.itwx = reinterpret_cast<const ulonglong2 *>(d_tables + (size_t)6 * P * N);
        ntt.tws = reinterpret_cast<const double *>(d_tables + (size_t)8 * P * N);
        ntt.itws = reinterpret_cast<const double *>(d_tables + (size_t)9 * P * N);
        ntt.logN = logN;

        std::vector<u64> pm(P);
        for (int p = 0; p < P; p++) {
            u64 q = primes[p], v = 1 % q;
            for (int k = 0; k < K; k++) v = h_mulm(v, primes[L + k] % q, q);
            pm[p] = v;
        }
        d_pmod = alloc(P);
        cuda_check(cudaMemcpyAsync(d_pmod, pm.data(), P * 8, cudaMemcpyHostToDevice, stream), "pmod");
        {
            // slot-wise multiplication by i is multiplication by X^(N/2); NTT
            // position t evaluates at psi^(2 brv(t) + 1), so the multiplier is
            // w = psi^(N/2) (w^2 = -1) for t < N/2 and -w above
            std::vector<u64> iu((size_t)4 * P);
            for (int p = 0; p < P; p++) {
                const u64 q = primes[p], w = h_powm(find_psi(q, logN), (u64)N / 2, q);
                iu[4 * p] = w, iu[4 * p + 1] = h_shoup(w, q);
                iu[4 * p + 2] = q - w, iu[4 * p + 3] = h_shoup(q - w, q);
            }
            d_iunit = alloc((size_t)4 * P);
            cuda_check(cudaMemcpyAsync(d_iunit, iu.data(), iu.size() * 8, cudaMemcpyHostToDevice, stream), "iunit");
            sync();
        }
        {
            std::vector<u64> cls((size_t)L * 9, 0);
            bsgs_mma_class_consts(cls.data(), primes.data(), L);
            d_cls8 = alloc((size_t)L * 9);
            cuda_check(cudaMemcpyAsync(d_cls8, cls.data(), cls.size() * 8, cudaMemcpyHostToDevice, stream), "cls8");
            d_tc_err = (int *)alloc(1);
            cuda_check(cudaMemsetAsync(d_tc_err, 0, 8, stream), "tc error word");
            const char *m = std::getenv("HELRM_B200_MAC");
            use_tc = m && std::string(m) == "tc";
        }

        build_level_tables();
        sync();
    }

    void build_level_tables() {
        lv.assign(L + 1, LevelTabs{});
        for (int nq = 1; nq <= L; nq++) {
            const int ne = nq + K, beta = beta_of(nq);
            std::vector<u64> qhinv((size_t)beta * alpha, 0), qhinvp((size_t)beta * alpha, 0);
            std::vector<u64> qhat((size_t)beta * alpha * ne, 0), qjneg((size_t)beta * ne, 0);
            for (int j = 0; j < beta; j++) {
                int lo = j * alpha, hi = std::min(lo + alpha, nq), na = hi - lo;
                for (int e = 0; e < ne; e++) {
                    int pe = e < nq ? e : L + (e - nq);
                    u64 t = primes[pe], v = 1 % t;
                    for (int m = 0; m < na; m++) v = h_mulm(v, primes[lo + m] % t, t);
                    qjneg[(size_t)j * ne + e] = v ? t - v : 0;
                }
                for (int m = 0; m < na; m++) {
                    u64 qm = primes[lo + m], v = 1 % qm;
                    for (int m2 = 0; m2 < na; m2++)
                        if (m2 != m) v = h_mulm(v, primes[lo + m2] % qm, qm);
                    qhinv[(size_t)j * alpha + m] = h_invm(v, qm);
                    qhinvp[(size_t)j * alpha + m] = h_shoup(qhinv[(size_t)j * alpha + m], qm);
                    for (int e = 0; e < ne; e++) {
                        int pe = e < nq ? e : L + (e - nq);
                        if (pe >= lo && pe < hi) continue;
                        u64 t = primes[pe], w = 1 % t;
                        for (int m2 = 0; m2 < na; m2++)
                            if (m2 != m) w = h_mulm(w, primes[lo + m2] % t, t);
                        qhat[((size_t)j * alpha + m) * ne + e] = w;
                    }
                }
            }
            std::vector<u64> phinv(K), phinvp(K), phat((size_t)K * nq), pinv(nq), pinvp(nq), pneg(nq);
            for (int k = 0; k < K; k++) {
                u64 pk = primes[L + k], v = 1 % pk;
                for (int k2 = 0; k2 < K; k2++)
                    if (k2 != k) v = h_mulm(v, primes[L + k2] % pk, pk);
                phinv[k] = h_invm(v, pk);
                phinvp[k] = h_shoup(phinv[k], pk);
                for (int i = 0; i < nq; i++) {
                    u64 q = primes[i], w = 1 % q;
                    for (int k2 = 0; k2 < K; k2++)
                        if (k2 != k) w = h_mulm(w, primes[L + k2] % q, q);
                    phat[(size_t)k * nq + i] = w;
                }
            }
            for (int i = 0; i < nq; i++) {
                u64 q = primes[i], v = 1 % q;
                for (int k = 0; k < K; k++) v = h_mulm(v, primes[L + k] % q, q);
                pinv[i] = h_invm(v, q);
                pinvp[i] = h_shoup(pinv[i], q);
                pneg[i] = v ? q - v : 0;
            }
            std::vector<u64> qlinv(nq, 0), qlinvp(nq, 0);
            if (nq >= 2) {
                u64 ql = primes[nq - 1];
                for (int i = 0; i < nq - 1; i++) {
                    qlinv[i] = h_invm(ql % primes[i], primes[i]);
                    qlinvp[i] = h_shoup(qlinv[i], primes[i]);
                }
            }
            std::vector<u64> blob;
            auto put = [&](const std::vector<u64> &v) {
                size_t off = blob.size();
                blob.insert(blob.end(), v.begin(), v.end());
                return off;
            };
            auto packed = [](std::vector<u64> v) {  // split-30 form: (v >> 30) << 32 | (v & (2^30 - 1))
                for (auto &x : v) x = ((x >> 30) << 32) | (x & ((1ull << 30) - 1));
                return v;
            };
            // q-row targets (primes below 2^40) as exact doubles: qhat as
            // pairs {t, fl(t / q_e)} (quotient estimates of the FP64 modular
            // products), qjneg as t; special-prime targets left zero
            auto pairs_d = [&](const std::vector<u64> &v) {
                std::vector<u64> o(2 * v.size(), 0);
                for (size_t i = 0; i < v.size(); i++) {
                    const int e = (int)(i % ne);
                    if (e >= nq || primes[e] >= (1ull << 40)) continue;
                    const double t = (double)v[i], r = t / (double)primes[e];
                    std::memcpy(&o[2 * i], &t, 8);
                    std::memcpy(&o[2 * i + 1], &r, 8);
                }
                return o;
            };
            auto singles_d = [&](const std::vector<u64> &v) {
                std::vector<u64> o(v.size(), 0);
                for (size_t i = 0; i < v.size(); i++) {
                    const int e = (int)(i % ne);
                    if (e >= nq || primes[e] >= (1ull << 40)) continue;
                    const double t = (double)v[i];
                    std::memcpy(&o[i], &t, 8);
                }
                return o;
            };
            size_t o_qhinv = put(qhinv), o_qhinvp = put(qhinvp), o_qhat = put(qhat), o_qjneg = put(qjneg),
                   o_pneg = put(pneg), o_qhat_s = put(packed(qhat)), o_qjneg_s = put(packed(qjneg));
            if (blob.size() & 1) blob.push_back(0);  // 16-byte alignment of the pairs
            size_t o_qhat_d = put(pairs_d(qhat)), o_qjneg_d = put(singles_d(qjneg));
            size_t o_phinv = put(phinv), o_phinvp = put(phinvp), o_phat = put(phat), o_pinv = put(pinv),
                   o_pinvp = put(pinvp), o_qlinv = put(qlinv), o_qlinvp = put(qlinvp), o_phat_s = put(packed(phat)),
                   o_pneg_s = put(packed(pneg));
            // split-30 basis conversion: every prime below 2^60, or main
            // primes below 2^40 with special primes below 2^61
            bool below60 = true, small_main = true, special61 = true;
            for (int i = 0; i < P; i++) below60 = below60 && primes[i] < (1ull << 60);
            for (int i = 0; i < L; i++) small_main = small_main && primes[i] < (1ull << 40);
            for (int i = L; i < P; i++) special61 = special61 && primes[i] < (1ull << 61);
            const bool split_ok = below60 || (small_main && special61);
            LevelTabs &T = lv[nq];
            T.blob = alloc(blob.size());
            cuda_check(cudaMemcpyAsync(T.blob, blob.data(), blob.size() * 8, cudaMemcpyHostToDevice, stream),
                       "level tables");
            T.beta = beta;
            T.mu.qhinv = T.blob + o_qhinv;
            T.mu.qhinvp = T.blob + o_qhinvp;
            T.mu.qhat = T.blob + o_qhat;
            T.mu.qjneg = T.blob + o_qjneg;
            T.mu.qhat_s = T.blob + o_qhat_s;
            T.mu.qjneg_s = T.blob + o_qjneg_s;
            T.mu.qhat_d = reinterpret_cast<const double2 *>(T.blob + o_qhat_d);
            T.mu.qjneg_d = reinterpret_cast<const double *>(T.blob + o_qjneg_d);
            T.mu.split = small_main && special61 ? 1 : split_ok ? 2 : 0;  // 2: some main prime of 2^40 or more
            T.md.pneg = T.blob + o_pneg;
            T.md.phat_s = T.blob + o_phat_s;
            T.md.pneg_s = T.blob + o_pneg_s;
            T.md.split = split_ok ? 1 : 0;
            T.md.phinv = T.blob + o_phinv;
            T.md.phinvp = T.blob + o_phinvp;
            T.md.phat = T.blob + o_phat;
            T.md.pinv = T.blob + o_pinv;
            T.md.pinvp = T.blob + o_pinvp;
            T.qlinv = T.blob + o_qlinv;
            T.qlinvp = T.blob + o_qlinvp;
        }
    }

    ~Context() {
        if (stream) {
            cudaStreamSynchronize(stream);
            if (up) {
                cudaStreamSynchronize(up);
                cudaStreamSynchronize(dn);
            }
            for (auto &kv : cts) release(kv.second.d);
            for (auto &kv : pts) release(kv.second.d);
            for (auto &kv : lts) free_lt(*kv.second);
            for (auto &kv : rot_keys) release(kv.second);
            release(d_rlk);
            release(d_sk);
            for (auto &t : lv) release(t.blob);
            for (auto &kv : tables) release(kv.second.tab);
            for (auto &kv : poly_plans) release(kv.second.d_consts);
            release(d_pmod);
            release(d_cls8);
            release(d_tc_err);
            release(d_iunit);
            release(d_enc_perm);
            release(d_enc_tw);
            release(d_tables);
            if (up) {
                cudaStreamSynchronize(up);
                cudaStreamSynchronize(dn);
            }
            cudaStreamSynchronize(stream);
            if (up) {
                cudaEventDestroy(ev_up);
                cudaEventDestroy(ev_dn);
                cudaEventDestroy(ev_comp);
                cudaStreamDestroy(up);
                cudaStreamDestroy(dn);
            }
            cudaStreamDestroy(stream);
        }
    }

    // ---------------------------------------------------------- registries
    int put_ct(const Ct &c) {
        int id = next_id++;
        cts[id] = c;
        return id;
    }
    int put_pt(const Pt &p) {
        int id = next_id++;
        pts[id] = p;
        return id;
    }
    Ct &ct(int id) {
        auto it = cts.find(id);
        if (it == cts.end()) HB_THROW(HB_ENOENT, "unknown ciphertext id " + std::to_string(id));
        return it->second;
    }
    Pt &pt(int id) {
        auto it = pts.find(id);
        if (it == pts.end()) HB_THROW(HB_ENOENT, "unknown plaintext id " + std::to_string(id));
        return it->second;
    }
    LinTrans &lt(int id) {
        auto it = lts.find(id);
        if (it == lts.end()) HB_THROW(HB_ENOENT, "unknown linear transform id " + std::to_string(id));
        return *it->second;
    }
    void del_ct(int id) {
        auto it = cts.find(id);
        if (it == cts.end()) return;
        release_ct(it->second);
        cts.erase(it);
    }
    void del_pt(int id) {
        auto it = pts.find(id);
        if (it == pts.end()) return;
        release(it->second.d);
        pts.erase(it);
    }
    void free_lt(LinTrans &t) {
        for (auto &kv : t.pts) release(kv.second.d);
        t.pts.clear();
        for (auto *p : t.plan_dev) release(p);
        t.plan_dev.clear();
    }
    // move the content of `from` into `id`
    void replace_ct(int id, int from) {
        Ct &dst = ct(id);
        Ct src = ct(from);
        release_ct(dst);
        dst = src;
        cts.erase(from);
    }

    Ct new_ct(int nq, int npoly, double scale) {
        Ct c;
        c.nq = nq;
        c.npoly = npoly;
        c.scale = scale;
        c.slots = slots;
        c.d = alloc((size_t)npoly * nq * N);
        return c;
    }
    int level_of(const Ct &c) const { return c.nq - 1; }

    // ---------------------------------------------------------- keys
    void require_sk() const {
        if (!d_sk) HB_THROW(HB_ESTATE, "secret key not generated (call GenerateSecretKey)");
    }

    void gen_secret() {
        // ternary secret of Hamming weight h (all coefficients when h >= N)
        std::vector<int8_t> s(N, 0);
        if (h >= N) {
            for (int n = 0; n < N; n++) s[n] = (hrand64(seed, DOM_SK_SIGN, n) >> 63) ? 1 : -1;
        } else {
            std::vector<unsigned> perm(N);
            for (int i = 0; i < N; i++) perm[i] = i;
            for (int i = 0; i < h; i++) {
                u64 r = hrand64(seed, DOM_SK_POS, i);
                unsigned j = i + (unsigned)(((hu128)r * (u64)(N - i)) >> 64);
                std::swap(perm[i], perm[j]);
                s[perm[i]] = (hrand64(seed, DOM_SK_SIGN, i) >> 63) ? 1 : -1;
            }
        }
        std::vector<u64> rows((size_t)P * N);
        for (int p = 0; p < P; p++)
            for (int n = 0; n < N; n++) rows[(size_t)p * N + n] = s[n] >= 0 ? (u64)s[n] : primes[p] - 1;
        if (!d_sk) d_sk = alloc((size_t)P * N);
        cuda_check(cudaMemcpyAsync(d_sk, rows.data(), rows.size() * 8, cudaMemcpyHostToDevice, stream), "sk");
        ntt_forward(d_sk, P, rowmap(P, L, L), ntt, stream);
        sync();
    }

    // switching key from `target` (NTT, [P][N]) to s
    u64 *gen_swk(const u64 *target, u64 kseed) {
        u64 *key = alloc(key_words());
        u64 *e = alloc((size_t)P * N);
        const RowMap all = rowmap(P, L, L);
        for (int j = 0; j < dnum; j++) {
            u64 *b = key + ((size_t)j * 2 + 0) * P * N;
            u64 *a = key + ((size_t)j * 2 + 1) * P * N;
            sample_uniform(a, P, nullptr, all, kseed, DOM_SWK_A, (u64)j * P * N, 0, logN, stream);
            sample_cbd(e, P, all, kseed, DOM_SWK_E, (u64)j * N, logN, stream);
            ntt_forward(e, P, all, ntt, stream);
            int lo = j * alpha, hi = std::min(lo + alpha, L);
            swk_combine(b, a, e, d_sk, target, d_pmod, P, lo, hi, logN, stream);
        }
        release(e);
        key_bytes += key_words() * 8;
        keygen_counter++;
        return key;
    }

    u64 galois_of(int k) const {
        int kn = ((k % slots) + slots) % slots;
        return h_powm(5, (u64)kn, 2ull * N);
    }

    u64 *rotation_key(u64 g) {
        auto it = rot_keys.find(g);
        if (it != rot_keys.end()) return it->second;
        require_sk();
        u64 *t = alloc((size_t)P * N);
        ew_automorphism(t, d_sk, P, g, logN, stream);
        u64 *key = gen_swk(t, hrand64(seed, DOM_KEYSEED, g));
        release(t);
        rot_keys[g] = key;
        return key;
    }

    void gen_relin() {
        require_sk();
        if (d_rlk) return;
        u64 *t = alloc((size_t)P * N);
        // s^2 over all primes: tensor-free elementwise square
        MacArgs m{};
        m.ct[0] = d_sk;
        m.pt[0] = d_sk;
        m.n = 1;
        // ew_mac treats rows as q rows of one poly; P rows map to primes 0..P-1
        ew_mac(t, m, 1, P, logN, stream);
        d_rlk = gen_swk(t, hrand64(seed, DOM_KEYSEED, 0));
        release(t);
    }

    // ---------------------------------------------------------- encode
    // integer coefficients -> NTT residues on `rows` rows (q rows then aux)
    // ---------------------------------------------------------- encoding on the device
    EncTables enc_tables_dev() {
        if (!d_enc_perm) {
            const size_t n = (size_t)N / 2;
            d_enc_perm = (int *)alloc((n + 1) / 2);
            d_enc_tw = (double2 *)alloc(n / 2 > 0 ? n : 2);  // n/2 entries of 16 bytes
            enc_tables(d_enc_perm, d_enc_tw, logN, stream);
        }
        return EncTables{d_enc_perm, d_enc_tw, logN};
    }
    // count vectors of nvals slot values (interleaved re, im when cplx) ->
    // plaintexts at dsts[v] ([nq (+K)][N], NTT order), scale `scale`
    void encode_device(const double *vals, int nvals, bool cplx, int count, int nq, bool ext, double scale,
                       u64 *const *dsts) {
        if (count <= 0) return;
        if (nvals < 0 || nvals > slots) HB_THROW(HB_EINVAL, "encode: more values than slots");
        const size_t per = (size_t)nvals * (cplx ? 2 : 1);
        // |coefficient| <= scale * max |slot| (the inverse transform averages)
        double mx = 0.0;
        for (size_t i = 0; i < per * count; i++) mx = std::max(mx, std::fabs(vals[i]));
        if (cplx) mx *= 2.0;
        if (!std::isfinite(mx) || !(mx * scale < 4.0e18))
            HB_THROW(HB_EINVAL, "encode: value * scale beyond 2^62 (or not finite)");
        const EncTables et = enc_tables_dev();
        const int rows = nq + (ext ? K : 0);
        const RowMap rm = rowmap(rows, nq, L);
        const int chunk = std::min(count, HB_PTR_BATCH);
        u64 *dv = alloc(std::max<size_t>(1, per * chunk));
        double2 *z = (double2 *)alloc((size_t)chunk * N);  // chunk x N/2 complex points
        for (int c0 = 0; c0 < count; c0 += chunk) {
            const int cnt = std::min(chunk, count - c0);
            if (per)
                cuda_check(cudaMemcpyAsync(dv, vals + per * c0, per * cnt * 8, cudaMemcpyHostToDevice, stream),
                           "encode values");
            enc_scatter(z, (const double *)dv, nvals, cplx ? 1 : 0, cnt, et, stream);
            enc_ifft(z, cnt, et, stream);
            PtrBatchW d{};
            for (int i = 0; i < cnt; i++) d.p[i] = dsts[c0 + i];
            enc_round(d, z, rows, rm, scale, cnt, et, stream);
            for (int i = 0; i < cnt; i++) ntt_forward(dsts[c0 + i], rows, rm, ntt, stream);
        }
        release(dv);
        release(z);
    }

    int encode(const double *inter, int n, int level, double scale, bool ext) {
        if (level < 0 || level >= L) HB_THROW(HB_EINVAL, "encode: level out of range");
        if (n > slots) HB_THROW(HB_EINVAL, "encode: more values than slots");
        if (!(scale > 0)) scale = default_scale;
        Pt p;
        p.nq = level + 1;
        p.ext = ext;
        p.scale = scale;
        p.slots = slots;
        p.d = alloc((size_t)(p.nq + (ext ? K : 0)) * N);
        encode_device(inter, n, true, 1, p.nq, ext, scale, &p.d);
        return put_pt(p);
    }

    // decode (NTT) plaintext rows -> interleaved values
    // the slots of plaintext rows d (nq limbs, NTT form) at `scale`, as
    // interleaved (re, im) pairs, decoded on the device: the inverse NTT of
    // the first min(nq, 4) limbs, the centred Garner CRT, the special FFT;
    // only the slot values cross to the host
    void decode_rows(const u64 *d, int nq, double scale, std::vector<double> &out) {
        const int nc = std::min(nq, HB_DEC_MAX);
        u64 *tmp = alloc((size_t)nc * N);
        d2d(tmp, d, (size_t)nc * N);
        ntt_inverse(tmp, nc, qmap(nc), ntt, stream);
        const CrtPlan plan(primes.data(), nc);
        DecCrt dc{};
        dc.n = nc;
        for (int i = 0; i < nc; i++) {
            dc.minv[i] = plan.minv[i];
            for (int k = 0; k < nc; k++) dc.mmod[i * HB_DEC_MAX + k] = plan.mmod[(size_t)i * nc + k];
        }
        u64 *coef = alloc(N), *z = alloc(N), *dv = alloc((size_t)2 * slots);
        decode_slots((double *)dv, tmp, dc, scale, 1, (double *)coef, (double2 *)z, enc_tables_dev(), stream);
        out.resize((size_t)2 * slots);
        cuda_check(cudaMemcpyAsync(out.data(), dv, out.size() * 8, cudaMemcpyDeviceToHost, stream), "decode");
        sync();
        release(tmp);
        release(coef);
        release(z);
        release(dv);
    }

    // ---------------------------------------------------------- encrypt
    Ct encrypt_rows(const u64 *m, int nq, double scale, u64 ct_seed) {
        require_sk();
        Ct c = new_ct(nq, 2, scale);
        u64 *c0 = c.d, *c1 = c.d + (size_t)nq * N;
        u64 *e = alloc((size_t)nq * N);
        sample_uniform(c1, nq, nullptr, qmap(nq), ct_seed, DOM_ENC_A, 0, 0, logN, stream);
        sample_cbd(e, nq, qmap(nq), ct_seed, DOM_ENC_E, 0, logN, stream);
        ntt_forward(e, nq, qmap(nq), ntt, stream);
        enc_combine(c0, c1, e, d_sk, m, nq, logN, stream);
        release(e);
        return c;
    }

    // ---------------------------------------------------------- batch packing
    // [nb][2][nq][N] <- the first nq rows of each ciphertext's two polys (one
    // launch per HB_PTR_BATCH ciphertexts)
    void gather_cts(u64 *dst, const std::vector<const Ct *> &v, int nq) {
        const size_t words = (size_t)nq * N;
        for (size_t b0 = 0; b0 < v.size(); b0 += HB_PTR_BATCH) {
            const int n = (int)std::min<size_t>(HB_PTR_BATCH, v.size() - b0);
            PtrBatch s0{}, s1{};
            for (int i = 0; i < n; i++) {
                s0.p[i] = v[b0 + i]->d;
                s1.p[i] = v[b0 + i]->d + (size_t)v[b0 + i]->nq * N;
            }
            gather_items(dst + b0 * 2 * words, s0, s1, 2, words, n, stream);
        }
    }
    // each destination <- its `words`-word item of the contiguous src
    void scatter_words(const std::vector<u64 *> &dsts, const u64 *src, size_t words) {
        for (size_t b0 = 0; b0 < dsts.size(); b0 += HB_PTR_BATCH) {
            const int n = (int)std::min<size_t>(HB_PTR_BATCH, dsts.size() - b0);
            PtrBatchW d{};
            for (int i = 0; i < n; i++) d.p[i] = dsts[b0 + i];
            scatter_items(d, src + b0 * words, words, n, stream);
        }
    }

    // ---------------------------------------------------------- key switching pieces
    // ModUp of nb polys (nq rows each, NTT) -> D [nb][beta][ne][N]
    void modup(u64 *D, const u64 *a, int nq, int nb, size_t a_stride) {
        const int ne = nq + K, beta = beta_of(nq);
        u64 *X = alloc((size_t)nb * nq * N);
        ntt_inverse_from(X, a, a_stride, nq, nb * nq, qmap(nq), ntt, stream);
        modup_bconv(D, X, a, nq, K, L, alpha, beta, lv[nq].mu, logN, nb, (size_t)nq * N, (size_t)beta * ne * N,
                    a_stride, stream);
        RowMap m = extmap(nq);
        m.alpha = alpha;
        m.ndig = beta;
        ntt_forward(D, nb * beta * ne, m, ntt, stream);
        release(X);
    }

    // ModDown of nb extended polys x (ne rows, item stride xs) -> out (nq rows, stride os),
    // optionally + addend[tau_g] (stride as) and + add2 (unrotated, stride a2s)
    void moddown(u64 *out, const u64 *x, int nq, int nb, size_t xs, size_t os, const u64 *addend = nullptr,
                 u64 add_g = 1, size_t as = 0, const u64 *add2 = nullptr, size_t a2s = 0) {
        u64 *Y = alloc((size_t)nb * K * N);
        RowMap pm = rowmap(K, 0, L);
        ntt_inverse_from(Y, x + (size_t)nq * N, xs, K, nb * K, pm, ntt, stream);
        u64 *Z = alloc((size_t)nb * nq * N);
        moddown_bconv(Z, Y, nq, K, L, lv[nq].md, logN, nb, (size_t)K * N, (size_t)nq * N, stream);
        ntt_forward(Z, nb * nq, qmap(nq), ntt, stream);
        moddown_combine(out, x, Z, nq, lv[nq].md, addend, add_g, logN, nb, xs, (size_t)nq * N, os, as, stream, add2,
                        a2s);
        release(Y);
        release(Z);
    }

    // rotations of nb ciphertexts (contiguous [nb][2][nq][N] at `in`) by
    // Galois g into `out` (same layout): one ModUp per ciphertext.  With
    // `fold`, out = in + rot(in) (the hybrid fold's step, added in the
    // ModDown combine; out must not alias in).
    void rotate_batch(u64 *out, const u64 *in, int nq, int nb, u64 g, const u64 *key, bool fold = false) {
        const int ne = nq + K, beta = beta_of(nq);
        const size_t cts_ = (size_t)2 * nq * N;
        u64 *D = alloc((size_t)nb * beta * ne * N);
        modup(D, in + (size_t)nq * N, nq, nb, cts_);
        u64 *acc = alloc((size_t)nb * 2 * ne * N);
        keymult(acc, D, key, g, nq, K, L, beta, P, nullptr, false, logN, nb, (size_t)beta * ne * N,
                (size_t)2 * ne * N, 0, stream);
        release(D);
        moddown(out, acc, nq, nb, (size_t)2 * ne * N, cts_, in, g, cts_, fold ? in : nullptr, cts_);
        moddown(out + (size_t)nq * N, acc + (size_t)ne * N, nq, nb, (size_t)2 * ne * N, cts_, nullptr, 1, 0,
                fold ? in + (size_t)nq * N : nullptr, cts_);
        release(acc);
    }

    // hoisted: one ciphertext, many Galois elements
    void rotate_hoisted(const u64 *in, int nq, int nb, const std::vector<u64> &gs, const std::vector<u64 *> &outs,
                        size_t out_stride) {
        const int ne = nq + K, beta = beta_of(nq);
        const size_t cts_ = (size_t)2 * nq * N;
        u64 *D = alloc((size_t)nb * beta * ne * N);
        modup(D, in + (size_t)nq * N, nq, nb, cts_);
        u64 *acc = alloc((size_t)nb * 2 * ne * N);
        for (size_t r = 0; r < gs.size(); r++) {
            u64 *key = rotation_key(gs[r]);
            keymult(acc, D, key, gs[r], nq, K, L, beta, P, nullptr, false, logN, nb, (size_t)beta * ne * N,
                    (size_t)2 * ne * N, 0, stream);
            moddown(outs[r], acc, nq, nb, (size_t)2 * ne * N, out_stride, in, gs[r], cts_);
            moddown(outs[r] + (size_t)nq * N, acc + (size_t)ne * N, nq, nb, (size_t)2 * ne * N, out_stride);
        }
        release(acc);
        release(D);
    }

    void relinearize(u64 *out, const u64 *in3, int nq) { relinearize_batch(out, in3, nq, 1); }

    // nb degree-2 ciphertexts [nb][3][nq][N] -> [nb][2][nq][N]
    void relinearize_batch(u64 *out, const u64 *in3, int nq, int nb) {
        const int ne = nq + K, beta = beta_of(nq);
        const size_t s3 = (size_t)3 * nq * N, s2 = (size_t)2 * nq * N;
        u64 *D = alloc((size_t)nb * beta * ne * N);
        modup(D, in3 + (size_t)2 * nq * N, nq, nb, s3);
        u64 *acc = alloc((size_t)nb * 2 * ne * N);
        keymult(acc, D, d_rlk, 1, nq, K, L, beta, P, nullptr, false, logN, nb, (size_t)beta * ne * N,
                (size_t)2 * ne * N, 0, stream);
        release(D);
        moddown(out, acc, nq, nb, (size_t)2 * ne * N, s2, in3, 1, s3);
        moddown(out + (size_t)nq * N, acc + (size_t)ne * N, nq, nb, (size_t)2 * ne * N, s2, in3 + (size_t)nq * N, 1,
                s3);
        release(acc);
    }

    // rescale nb ciphertexts [nb][npoly][nq] -> [nb][npoly][nq-1]
    void rescale(u64 *out, const u64 *in, int npoly, int nq, int nb, size_t in_stride, size_t out_stride) {
        if (nq < 2) HB_THROW(HB_ESTATE, "rescale: ciphertext already at level 0");
        const int l = nq - 1;
        u64 *R = alloc((size_t)nb * npoly * N);
        for (int pl = 0; pl < npoly; pl++)
            copy_strided(R + (size_t)pl * N, (size_t)npoly * N, in + ((size_t)pl * nq + l) * N, in_stride, N, nb,
                         stream);
        RowMap rm = rowmap(1, 1, L);
        rm.pbase = l;
        ntt_inverse(R, nb * npoly, rm, ntt, stream);
        u64 *W = alloc((size_t)nb * npoly * l * N);
        rescale_prep(W, R, npoly, l, primes[l], logN, nb, (size_t)npoly * N, (size_t)npoly * l * N, stream);
        ntt_forward(W, nb * npoly * l, qmap(l), ntt, stream);
        rescale_combine(out, in, W, npoly, nq, lv[nq].qlinv, lv[nq].qlinvp, logN, nb, in_stride,
                        (size_t)npoly * l * N, out_stride, stream);
        release(R);
        release(W);
    }
    // the same rescale with both temporaries carved from caller-owned
    // scratch of nb*npoly*nq*N words (R first, then W); nothing is allocated
    void rescale_scratch(u64 *out, const u64 *in, int npoly, int nq, int nb, size_t in_stride,
                         size_t out_stride, u64 *scratch) {
        if (nq < 2) HB_THROW(HB_ESTATE, "rescale: ciphertext already at level 0");
        const int l = nq - 1;
        u64 *R = scratch;
        u64 *W = scratch + (size_t)nb * npoly * N;
        for (int pl = 0; pl < npoly; pl++)
            copy_strided(R + (size_t)pl * N, (size_t)npoly * N, in + ((size_t)pl * nq + l) * N, in_stride, N, nb,
                         stream);
        RowMap rm = rowmap(1, 1, L);
        rm.pbase = l;
        ntt_inverse(R, nb * npoly, rm, ntt, stream);
        rescale_prep(W, R, npoly, l, primes[l], logN, nb, (size_t)npoly * N, (size_t)npoly * l * N, stream);
        ntt_forward(W, nb * npoly * l, qmap(l), ntt, stream);
        rescale_combine(out, in, W, npoly, nq, lv[nq].qlinv, lv[nq].qlinvp, logN, nb, in_stride,
                        (size_t)npoly * l * N, out_stride, stream);
    }

    // ---------------------------------------------------------- bootstrapping: ModRaise
    // a level-0 ciphertext (one limb, NTT) -> every main prime: each
    // coefficient of c0, c1 is lifted centred from q_0 and reduced modulo
    // q_i, so the result decrypts to m + q_0 I with I small (the integer
    // overflow of c0 + c1 s over q_0)
    int mod_raise(int id) {
        const Ct &x = ct(id);
        if (x.npoly != 2) HB_THROW(HB_ESTATE, "ModRaise: relinearize first");
        if (x.nq != 1) HB_THROW(HB_ESTATE, "ModRaise: the input must be at level 0");
        Ct o = new_ct(L, 2, x.scale);
        o.slots = x.slots;
        u64 *co = alloc((size_t)2 * N);
        d2d(co, x.d, (size_t)2 * N);
        RowMap r0 = rowmap(1, 1, L);
        ntt_inverse(co, 2, r0, ntt, stream);
        mod_raise_rows(o.d, co, L, logN, stream);
        ntt_forward(o.d, 2 * L, qmap(L), ntt, stream);
        release(co);
        return put_ct(o);
    }

    // ---------------------------------------------------------- level / scale alignment
    Ct drop_to(const Ct &c, int nq) {
        Ct o = new_ct(nq, c.npoly, c.scale);
        o.slots = c.slots;
        for (int pl = 0; pl < c.npoly; pl++)
            d2d(o.d + (size_t)pl * nq * N, c.d + (size_t)pl * c.nq * N, (size_t)nq * N);
        return o;
    }

    // absorbs scale drift below 1e-4 relative like the reference
    // (cheddar_pybind.cu:277-307); larger mismatches are errors.
    void check_scales(double a, double b, const char *op) {
        double diff = std::fabs(a - b);
        if (diff < 1e-12 * a) return;
        if (!(diff < 1e-4 * a))
            HB_THROW(HB_ESTATE, std::string(op) + ": scale mismatch beyond drift tolerance (" + std::to_string(a) +
                                    " vs " + std::to_string(b) + ")");
    }

    int add_sub(int a, int b, bool sub) {
        const Ct &ca = ct(a), &cb = ct(b);
        if (ca.npoly != cb.npoly) HB_THROW(HB_ESTATE, "add: ciphertext degrees differ");
        check_scales(ca.scale, cb.scale, sub ? "SubCiphertextNew" : "AddCiphertextNew");
        int nq = std::min(ca.nq, cb.nq);
        Ct o = new_ct(nq, ca.npoly, ca.scale);
        o.slots = std::max(ca.slots, cb.slots);
        for (int pl = 0; pl < ca.npoly; pl++) {
            if (sub)
                ew_sub(o.d + (size_t)pl * nq * N, ca.d + (size_t)pl * ca.nq * N, cb.d + (size_t)pl * cb.nq * N, nq,
                       qmap(nq), logN, stream);
            else
                ew_add(o.d + (size_t)pl * nq * N, ca.d + (size_t)pl * ca.nq * N, cb.d + (size_t)pl * cb.nq * N, nq,
                       qmap(nq), logN, stream);
        }
        return put_ct(o);
    }

    // constant value per prime (signed integer v, possibly beyond 64 bits)
    std::vector<u64> const_residues(long double v) {
        long double r = v >= 0 ? floorl(v + 0.5L) : -floorl(-v + 0.5L);
        if (!(fabsl(r) < 1.6e38L)) HB_THROW(HB_EINVAL, "scalar too large to encode");
        hi128 x = (hi128)r;
        std::vector<u64> res(P);
        for (int p = 0; p < P; p++) {
            u64 q = primes[p];
            if (x >= 0)
                res[p] = (u64)((hu128)x % q);
            else {
                u64 m = (u64)((hu128)(-x) % q);
                res[p] = m ? q - m : 0;
            }
        }
        return res;
    }

    int scalar_op(int id, long double value, int kind) {  // 0 add, 1 sub, 2 mul(int), 3 mul(float)
        const Ct &c = ct(id);
        Ct o = new_ct(c.nq, c.npoly, c.scale);
        o.slots = c.slots;
        std::vector<u64> res;
        if (kind == 0 || kind == 1) res = const_residues(value * (long double)c.scale);
        else if (kind == 2) res = const_residues(value);
        else res = const_residues(value * (long double)c.scale);
        if (kind == 1)
            for (int p = 0; p < P; p++) res[p] = res[p] ? primes[p] - res[p] : 0;
        ConstWords cw{};
        for (int p = 0; p < P; p++) {
            cw.v[p] = res[p];
            cw.vp[p] = h_shoup(res[p], primes[p]);
        }
        if (kind <= 1) {
            ew_add_const(o.d, c.d, cw, c.nq, qmap(c.nq), logN, stream);
            if (c.npoly > 1) d2d(o.d + (size_t)c.nq * N, c.d + (size_t)c.nq * N, (size_t)(c.npoly - 1) * c.nq * N);
        } else {
            ew_mul_const(o.d, c.d, cw, c.npoly * c.nq, qmap(c.nq), logN, stream);
            if (kind == 3) o.scale = c.scale * c.scale;
        }
        return put_ct(o);
    }

    int mul_plain(int ctid, int ptid) {
        const Ct &c = ct(ctid);
        const Pt &p = pt(ptid);
        int nq = std::min(c.nq, p.nq);
        Ct o = new_ct(nq, c.npoly, c.scale * p.scale);
        o.slots = c.slots;
        for (int pl = 0; pl < c.npoly; pl++)
            ew_mul_bcast(o.d + (size_t)pl * nq * N, c.d + (size_t)pl * c.nq * N, p.d, 1, nq, 0, logN, stream);
        return put_ct(o);
    }

    int add_plain(int ctid, int ptid, bool sub) {
        const Ct &c = ct(ctid);
        Pt p = pt(ptid);
        int tmp_pt = 0;
        if (std::fabs(p.scale - c.scale) > 1e-12 * c.scale) {
            // re-encode the plaintext at the ciphertext's scale (cheddar_pybind.cu:775-788)
            std::vector<double> vals;
            decode_rows(p.d, p.nq, p.scale, vals);
            tmp_pt = encode(vals.data(), slots, p.nq - 1, c.scale, false);
            p = pt(tmp_pt);
        }
        int nq = std::min(c.nq, p.nq);
        Ct o = new_ct(nq, c.npoly, c.scale);
        o.slots = c.slots;
        if (sub)
            ew_sub(o.d, c.d, p.d, nq, qmap(nq), logN, stream);
        else
            ew_add(o.d, c.d, p.d, nq, qmap(nq), logN, stream);
        for (int pl = 1; pl < c.npoly; pl++) d2d(o.d + (size_t)pl * nq * N, c.d + (size_t)pl * c.nq * N, (size_t)nq * N);
        if (tmp_pt) del_pt(tmp_pt);
        return put_ct(o);
    }

    int mac(const std::vector<int> &cids, const std::vector<int> &pids) {
        if (cids.empty() || cids.size() != pids.size())
            HB_THROW(HB_EINVAL, "MulPlaintextAccumNew: ct_ids/pt_ids must be equal-length and non-empty");
        int nq = 1 << 30;
        for (int id : cids) nq = std::min(nq, ct(id).nq);
        for (int id : pids) nq = std::min(nq, pt(id).nq);
        const double s0 = ct(cids[0]).scale * pt(pids[0]).scale;
        int sl = 0;
        for (size_t i = 0; i < cids.size(); i++) {
            const Ct &c = ct(cids[i]);
            if (c.npoly != 2) HB_THROW(HB_ESTATE, "MulPlaintextAccumNew: operand is degree-2; relinearize first");
            double s = c.scale * pt(pids[i]).scale;
            if (std::fabs(s - s0) > 1e-9 * s0)
                HB_THROW(HB_ESTATE, "MulPlaintextAccumNew: inconsistent ct*pt scale products across pairs");
            sl = std::max(sl, c.slots);
        }
        Ct o = new_ct(nq, 2, s0);
        o.slots = sl;
        // operands at a higher level are used through their first nq rows
        std::vector<u64 *> tmps;
        size_t done = 0;
        u64 *acc = nullptr;
        while (done < cids.size()) {
            size_t n = std::min((size_t)HB_MAC_MAX, cids.size() - done);
            MacArgs m{};
            for (size_t t = 0; t < n; t++) {
                const Ct &c = ct(cids[done + t]);
                const u64 *src = c.d;
                if (c.nq != nq) {
                    Ct dd = drop_to(c, nq);
                    tmps.push_back(dd.d);
                    src = dd.d;
                }
                m.ct[t] = src;
                m.pt[t] = pt(pids[done + t]).d;
            }
            m.n = (int)n;
            if (!acc) {
                ew_mac(o.d, m, 2, nq, logN, stream);
                acc = o.d;
            } else {
                u64 *part = alloc((size_t)2 * nq * N);
                ew_mac(part, m, 2, nq, logN, stream);
                ew_add(o.d, o.d, part, 2 * nq, qmap(nq), logN, stream);
                release(part);
            }
            done += n;
        }
        for (auto *p : tmps) release(p);
        return put_ct(o);
    }

    // ---------------------------------------------------------- broadcast constants and tables
    int encode_constant(double v, int level, double sc) {
        if (level < 0 || level >= L) HB_THROW(HB_EINVAL, "EncodeConstantNew: level out of range");
        const long double x = (long double)v * (long double)sc;
        if (!(std::fabs((double)x) < 9.2e18)) HB_THROW(HB_EINVAL, "EncodeConstantNew: scalar * scale beyond 2^63");
        const long long r = std::llroundl(x);
        Konst k;
        k.level = level;
        k.scale = sc;
        for (int i = 0; i <= level; i++) {
            const long long m = (long long)(r % (long long)primes[i]);
            k.words.push_back((u64)(m < 0 ? m + (long long)primes[i] : m));
        }
        const int id = next_id++;
        konsts[id] = std::move(k);
        return id;
    }
    const Konst &konst(int id) {
        auto it = konsts.find(id);
        if (it == konsts.end()) HB_THROW(HB_ENOENT, "constant " + std::to_string(id) + " not found");
        return it->second;
    }
    Table &table(int id) {
        auto it = tables.find(id);
        if (it == tables.end()) HB_THROW(HB_ENOENT, "table " + std::to_string(id) + " not found");
        return it->second;
    }
    int pack_constant_table(const int *ids, int n, int rows) {
        if (rows <= 0 || n <= 0 || n % rows) HB_THROW(HB_EINVAL, "PackConstantTableNew: ids must be a non-empty rows x cols table");
        Table t;
        t.rows = rows;
        t.cols = n / rows;
        const Konst &k0 = konst(ids[0]);
        t.level = k0.level;
        t.scale = k0.scale;
        const int nq = t.level + 1;
        std::vector<double> h((size_t)nq * n);
        for (int i = 0; i < n; i++) {
            const Konst &k = konst(ids[i]);
            if (k.level != t.level) HB_THROW(HB_EINVAL, "PackConstantTableNew: all constants must share one level");
            if (std::fabs(k.scale - t.scale) > 1e-9 * t.scale)
                HB_THROW(HB_EINVAL, "PackConstantTableNew: all constants must share one scale");
            for (int e = 0; e < nq; e++) h[(size_t)e * n + i] = (double)k.words[e];
        }
        t.tab = (double *)alloc(h.size());
        cuda_check(cudaMemcpyAsync(t.tab, h.data(), h.size() * 8, cudaMemcpyHostToDevice, stream), "table");
        sync();
        const int id = next_id++;
        tables[id] = std::move(t);
        return id;
    }
    int pack_plaintext_table(const int *ids, int n, int rows) {
        if (rows <= 0 || n <= 0 || n % rows) HB_THROW(HB_EINVAL, "PackPlaintextTableNew: ids must be a non-empty rows x cols table");
        Table t;
        t.rows = rows;
        t.cols = n / rows;
        t.pt = true;
        const Pt &p0 = pt(ids[0]);
        t.level = p0.nq - 1;
        t.scale = p0.scale;
        for (int i = 0; i < n; i++) {
            const Pt &p = pt(ids[i]);
            if (p.nq != p0.nq) HB_THROW(HB_EINVAL, "PackPlaintextTableNew: all plaintexts must share one level");
            if (std::fabs(p.scale - t.scale) > 1e-9 * t.scale)
                HB_THROW(HB_EINVAL, "PackPlaintextTableNew: all plaintexts must share one scale");
            t.pt_ids.push_back(ids[i]);
        }
        const int id = next_id++;
        tables[id] = std::move(t);
        return id;
    }
    void delete_table(int id) {
        Table &t = table(id);
        if (t.tab) release(t.tab);
        tables.erase(id);
    }
    // rows new ciphertexts: sum_k T[r][k] * ct_k at the table's level
    std::vector<int> table_matmul_ids(const int *cts, int n, Table &t) {
        if (n != t.cols)
            HB_THROW(HB_EINVAL, "table product: expected " + std::to_string(t.cols) + " ciphertexts, got " +
                                    std::to_string(n));
        const int nq = t.level + 1;
        double cscale = 0.0;
        std::vector<const u64 *> xp((size_t)2 * n);
        for (int k = 0; k < n; k++) {
            const Ct &c = ct(cts[k]);
            if (c.npoly != 2) HB_THROW(HB_ESTATE, "table product: operand is degree-2; relinearize first");
            if (c.nq < nq)
                HB_THROW(HB_ESTATE, "table product: ciphertext at level " + std::to_string(c.nq - 1) +
                                        " is below the table's level " + std::to_string(t.level));
            if (k == 0) cscale = c.scale;
            else if (std::fabs(c.scale - cscale) > 1e-9 * cscale)
                HB_THROW(HB_ESTATE, "table product: inconsistent ciphertext scales");
            xp[2 * k] = c.d;
            xp[2 * k + 1] = c.d + (size_t)c.nq * N;
        }
        std::vector<int> outs;
        std::vector<u64 *> op;
        for (int r = 0; r < t.rows; r++) {
            Ct o = new_ct(nq, 2, cscale * t.scale);
            o.slots = ct(cts[0]).slots;
            op.push_back(o.d);
            outs.push_back(put_ct(o));
        }
        std::vector<const u64 *> pp;
        if (t.pt)
            for (int id : t.pt_ids) pp.push_back(pt(id).d);
        // pointer arrays in device memory, freed behind the launch
        u64 *dx = alloc(xp.size()), *dout = alloc(op.size()), *dpt = pp.empty() ? nullptr : alloc(pp.size());
        cuda_check(cudaMemcpyAsync(dx, xp.data(), xp.size() * 8, cudaMemcpyHostToDevice, stream), "matmul ptrs");
        cuda_check(cudaMemcpyAsync(dout, op.data(), op.size() * 8, cudaMemcpyHostToDevice, stream), "matmul ptrs");
        if (dpt) cuda_check(cudaMemcpyAsync(dpt, pp.data(), pp.size() * 8, cudaMemcpyHostToDevice, stream), "matmul ptrs");
        MatMulArgs a{};
        a.out = (u64 *const *)dout;
        a.x = (const u64 *const *)dx;
        a.tab = t.tab;
        a.pts = (const u64 *const *)dpt;
        a.rows = t.rows;
        a.cols = t.cols;
        a.nq = nq;
        a.logN = logN;
        table_matmul(a, t.pt, stream);
        release(dx);
        release(dout);
        if (dpt) release(dpt);
        sync();  // the host pointer arrays above go out of scope
        return outs;
    }

    // ---------------------------------------------------------- linear transforms
    int generate_lt(const int *idxs, int n, const double *data, int width, int level, double ratio,
                    bool cplx = false, double pscale = 0.0) {
        if (n <= 0) HB_THROW(HB_EINVAL, "GenerateLinearTransform: no diagonals");
        if (width <= 0 || width > slots) HB_THROW(HB_EINVAL, "GenerateLinearTransform: bad diagonal width");
        if (level < 0 || level >= L) HB_THROW(HB_EINVAL, "GenerateLinearTransform: level out of range");
        // the diagonals at the level's prime, as the reference's Lattigo
        // backend encodes them (lineartransform.go:65): the rescale after
        // the transform divides that prime back out, so the output keeps
        // the input's scale exactly
        if (!(pscale > 0)) pscale = (double)primes[level];
        auto t = std::make_unique<LinTrans>();
        t->level = level;
        t->scale = pscale;
        t->use_bsgs = ratio > 0 && n > 1;
        int bs;
        const char *env = std::getenv("HELRM_B200_BS");
        if (t->use_bsgs) {
            bs = std::max(1, (int)std::ceil(std::sqrt((double)n * ratio)));
            if (env && *env) bs = std::max(1, std::atoi(env));
        } else {
            bs = slots;  // one giant group: every diagonal is a baby step
        }
        t->bs = bs;
        std::set<int> seen;
        for (int i = 0; i < n; i++) {
            int k = idxs[i];
            if (k < 0 || k >= slots) HB_THROW(HB_EINVAL, "GenerateLinearTransform: diagonal index out of range");
            if (!seen.insert(k).second) HB_THROW(HB_EINVAL, "GenerateLinearTransform: duplicate diagonal index");
            t->ks.push_back(k);
        }
        // encode every diagonal once (pre-rolled by g*bs), on the device in
        // batches of up to HB_PTR_BATCH diagonals
        std::vector<double> rolled;
        std::vector<u64 *> dsts;
        for (int i0 = 0; i0 < n; i0 += HB_PTR_BATCH) {
            const int cnt = std::min(HB_PTR_BATCH, n - i0);
            const int per = cplx ? 2 : 1;
            rolled.assign((size_t)cnt * width * per, 0.0);
            dsts.clear();
            for (int j = 0; j < cnt; j++) {
                const int i = i0 + j, k = idxs[i], g = t->use_bsgs ? k / bs : 0, shift = g * bs;
                const double *vals = data + (size_t)i * width * per;
                double *dst = &rolled[(size_t)j * width * per];
                for (int s = 0; s < width; s++) {
                    // numpy roll to the right by shift over the diagonal's own width
                    const int src = ((s - shift) % width + width) % width;
                    for (int e = 0; e < per; e++) dst[per * s + e] = vals[per * src + e];
                }
                Pt p;
                p.nq = level + 1;
                p.ext = true;
                p.scale = pscale;
                p.slots = slots;
                p.d = alloc((size_t)(p.nq + K) * N);
                t->pts[k] = p;
                dsts.push_back(p.d);
                const int b = t->use_bsgs ? k % bs : k;
                t->groups[g].push_back({b, k});
            }
            encode_device(rolled.data(), width, cplx, cnt, level + 1, true, pscale, dsts.data());
        }
        int id = next_id++;
        lts[id] = std::move(t);
        return id;
    }

    std::vector<int> lt_rotation_keys(const LinTrans &t) {
        std::set<int> d;
        for (auto &kv : t.groups) {
            int g = kv.first;
            for (auto &bk : kv.second)
                if (bk.first != 0) d.insert(bk.first);
            if (g != 0) d.insert(g * t.bs);
        }
        return std::vector<int>(d.begin(), d.end());
    }

    void build_plan(LinTrans &t, int nq) {
        if (t.plan_keygen == keygen_counter && t.plan_nq == nq) return;
        for (auto *p : t.plan_dev) release(p);
        t.plan_dev.clear();
        t.plan_chunks.clear();
        t.giant_of_slot.clear();
        for (auto &kv : t.groups) t.giant_of_slot.push_back(kv.first);
        const int nslots = (int)t.giant_of_slot.size();
        for (int s0 = 0; s0 < nslots; s0 += HB_GCH) {
            const int cnt = std::min(HB_GCH, nslots - s0);
            std::map<int, BabyDesc> babies;
            for (int gi = 0; gi < cnt; gi++) {
                int g = t.giant_of_slot[s0 + gi];
                for (auto &bk : t.groups[g]) {
                    int b = bk.first;
                    auto it = babies.find(b);
                    if (it == babies.end()) {
                        BabyDesc bd{};
                        if (b == 0) {
                            bd.galois = 1;
                            bd.key = nullptr;
                        } else {
                            bd.galois = galois_of(b);
                            auto kit = rot_keys.find(bd.galois);
                            if (kit == rot_keys.end()) bd.key = rotation_key(bd.galois);
                            else bd.key = kit->second;
                        }
                        it = babies.emplace(b, bd).first;
                    }
                    it->second.pt[gi] = t.pts[bk.second].d;
                }
            }
            std::vector<BabyDesc> all;
            for (auto &kv : babies) all.push_back(kv.second);
            // babies in groups of HB_BCH; later groups accumulate into the
            // inner sums the first group wrote
            for (size_t b0 = 0; b0 < all.size(); b0 += HB_BCH) {
                std::vector<BabyDesc> host(all.begin() + b0,
                                           all.begin() + std::min(all.size(), b0 + (size_t)HB_BCH));
                BabyDesc *dev = (BabyDesc *)alloc(host.size() * sizeof(BabyDesc) / 8 + 1);
                cuda_check(cudaMemcpyAsync(dev, host.data(), host.size() * sizeof(BabyDesc),
                                           cudaMemcpyHostToDevice, stream),
                           "plan");
                t.plan_dev.push_back(dev);
                BsgsChunk ch;
                ch.babies = dev;
                ch.nbabies = (int)host.size();
                ch.gbase = s0;
                ch.gcount = cnt;
                ch.nkeys = 0;
                ch.npts = 0;
                ch.accumulate = b0 > 0;
                for (auto &bd : host) {
                    ch.nkeys += bd.key != nullptr;
                    for (int gi = 0; gi < HB_GCH; gi++) ch.npts += bd.pt[gi] != nullptr;
                }
                ch.ptp = nullptr;
                if (use_tc && bsgs_mma_supported(nq, beta_of(nq))) {
                    // the chunk's plaintexts as byte planes for the tensor-core MAC
                    u64 *planes = alloc((bsgs_mma_planes_bytes(nq, logN) + 7) / 8);
                    t.plan_dev.push_back((BabyDesc *)planes);
                    ch.ptp = (const uint8_t *)planes;
                    bsgs_mma_planes((uint8_t *)planes, ch, nq, logN, stream);
                }
                t.plan_chunks.push_back(ch);
                sync();
            }
        }
        // giant keys
        for (int g : t.giant_of_slot)
            if (g != 0) rotation_key(galois_of(g * t.bs));
        t.plan_keygen = keygen_counter;
        t.plan_nq = nq;
    }

    // Double-hoisted BSGS over nb ciphertexts packed at `in` ([nb][2][nq][N]);
    // output [nb][2][nq][N] at `out`, scale ct*pt, not rescaled.
    void lt_eval_packed(LinTrans &t, const u64 *in, int nq, int nb, u64 *out) {
        build_plan(t, nq);
        const int ne = nq + K, beta = beta_of(nq);
        const size_t cts_ = (size_t)2 * nq * N, es = (size_t)ne * N;
        const int nslots = (int)t.giant_of_slot.size();
        u64 *D = alloc((size_t)nb * beta * es);
        modup(D, in + (size_t)nq * N, nq, nb, cts_);
        u64 *inner = alloc((size_t)nb * nslots * 2 * es);
        for (auto &ch : t.plan_chunks) {
            if (ch.ptp) {
                // q rows on the tensor cores, special rows on the CUDA cores
                bsgs_baby_mma(inner, in, D, ch, d_cls8, nq, K, L, beta, P, d_pmod, logN, nb, cts_, (size_t)beta * es,
                              (size_t)nslots * 2 * es, d_tc_err, stream);
                bsgs_baby_mac_special(inner, in, D, ch, nq, K, L, beta, P, t.level + 1, d_pmod, logN, nb, cts_,
                                      (size_t)beta * es, (size_t)nslots * 2 * es, stream);
            } else {
                // ciphertexts in chunks: one limb's rotated-digit gather set for
                // the chunk (chunk x (beta + 1) rows) stays L2-resident across the
                // waves of blocks, at the price of the chunk's keys and
                // plaintexts streaming once per chunk
                const int cc = mac_ct_chunk();
                for (int c0 = 0; c0 < nb; c0 += cc) {
                    const int n = std::min(cc, nb - c0);
                    bsgs_baby_mac(inner + (size_t)c0 * nslots * 2 * es, in + (size_t)c0 * cts_,
                                  D + (size_t)c0 * beta * es, ch, nq, K, L, beta, P, t.level + 1, d_pmod, logN, n,
                                  cts_, (size_t)beta * es, (size_t)nslots * 2 * es, stream);
                }
            }
        }
        release(D);
        // the giant-0 slot needs no rotation: its inner sum is the accumulator
        // itself (no copy); without one, a zeroed accumulator of its own
        int s0 = -1;
        for (int s = 0; s < nslots; s++)
            if (t.giant_of_slot[s] == 0) s0 = s;
        u64 *acc_own = nullptr, *acc;
        size_t acc_stride;
        if (s0 >= 0) {
            acc = inner + (size_t)s0 * 2 * es;
            acc_stride = (size_t)nslots * 2 * es;
        } else {
            acc_own = alloc((size_t)nb * 2 * es);
            zero(acc_own, (size_t)nb * 2 * es);
            acc = acc_own;
            acc_stride = 2 * es;
        }
        u64 *aq = alloc((size_t)nb * nq * N);
        std::vector<int> gslots;
        for (int s = 0; s < nslots; s++)
            if (t.giant_of_slot[s] != 0) gslots.push_back(s);
        // four digits: the giant steps in groups of up to lt_group(), one key
        // multiplication per group (the accumulator read and written once)
        const int G = (beta == 4 && logN >= 8) ? std::max(1, std::min(lt_group(), (int)gslots.size())) : 1;
        std::vector<u64 *> D2(G);
        for (auto &d : D2) d = alloc((size_t)nb * beta * es);
        const size_t is = (size_t)nslots * 2 * es;
        for (size_t i = 0; i < gslots.size();) {
            const int n = (int)std::min<size_t>(G, gslots.size() - i);
            const u64 *Dp[HB_MAX_GIANTS], *kp[HB_MAX_GIANTS], *ap[HB_MAX_GIANTS];
            u64 gp[HB_MAX_GIANTS];
            for (int k = 0; k < n; k++) {
                const int sl = gslots[i + k];
                gp[k] = galois_of(t.giant_of_slot[sl] * t.bs);
                kp[k] = rot_keys.at(gp[k]);
                ap[k] = inner + (size_t)sl * 2 * es;
                Dp[k] = D2[k];
                moddown(aq, inner + (size_t)sl * 2 * es + es, nq, nb, is, (size_t)nq * N);
                modup(D2[k], aq, nq, nb, (size_t)nq * N);
            }
            if (n >= 2)
                keymult_group(acc, n, Dp, kp, gp, ap, nq, K, L, beta, P, true, logN, nb, (size_t)beta * es, acc_stride,
                              is, stream);
            else
                keymult(acc, D2[0], kp[0], gp[0], nq, K, L, beta, P, ap[0], true, logN, nb, (size_t)beta * es,
                        acc_stride, is, stream);
            i += n;
        }
        release(aq);
        for (auto *d : D2) release(d);
        moddown(out, acc, nq, nb, acc_stride, cts_);
        moddown(out + (size_t)nq * N, acc + es, nq, nb, acc_stride, cts_);
        release(inner);
        if (acc_own) release(acc_own);
    }

    // giant steps per key multiplication in the LT (four digits)
    static int lt_group() { return HB_LT_GIANT_GROUP; }
    // ciphertexts per launch of the CUDA-core baby-step MAC
    static int mac_ct_chunk() {
        static int v = [] {
            const char *e = std::getenv("HELRM_B200_MAC_CHUNK");
            const int x = e && *e ? std::atoi(e) : HB_MAC_CT_CHUNK;
            return x > 0 ? x : HB_MAC_CT_CHUNK;
        }();
        return v;
    }
    size_t lt_bytes_per_ct(const LinTrans &t, int nq) {
        const int ne = nq + K, beta = beta_of(nq);
        const size_t es = (size_t)ne * N * 8;
        // inner sums, the digits of the baby steps or of one giant group
        // (and ModUp's temporaries), the accumulator, ModDown's temporaries
        return (size_t)t.groups.size() * 2 * es + (size_t)(lt_group() + 2) * beta * es + 2 * es +
               (size_t)6 * nq * N * 8;
    }

    void eval_lt_batch(int ltid, const std::vector<int> &ids, std::vector<int> &outs) {
        LinTrans &t = lt(ltid);
        outs.assign(ids.size(), 0);
        // group ciphertexts by the level they run at
        std::map<int, std::vector<size_t>> bylevel;
        for (size_t i = 0; i < ids.size(); i++) {
            const Ct &c = ct(ids[i]);
            if (c.npoly != 2) HB_THROW(HB_ESTATE, "EvaluateLinearTransform: input is degree-2; relinearize first");
            bylevel[std::min(c.nq, t.level + 1)].push_back(i);
        }
        size_t free_b = 0, tot_b = 0;
        cudaMemGetInfo(&free_b, &tot_b);
        for (auto &kv : bylevel) {
            const int nq = kv.first;
            const auto &idx = kv.second;
            size_t per = lt_bytes_per_ct(t, nq);
            size_t budget = std::min<size_t>(free_b / 2, (size_t)64 << 30);
            int chunk = (int)std::max<size_t>(1, std::min<size_t>(idx.size(), budget / std::max<size_t>(per, 1)));
            const size_t cts_ = (size_t)2 * nq * N;
            for (size_t c0 = 0; c0 < idx.size(); c0 += chunk) {
                int nb = (int)std::min<size_t>(chunk, idx.size() - c0);
                u64 *in = alloc((size_t)nb * cts_);
                std::vector<const Ct *> src(nb);
                for (int b = 0; b < nb; b++) src[b] = &ct(ids[idx[c0 + b]]);
                gather_cts(in, src, nq);
                u64 *out = alloc((size_t)nb * cts_);
                lt_eval_packed(t, in, nq, nb, out);
                release(in);
                std::vector<u64 *> dst(nb);
                for (int b = 0; b < nb; b++) {
                    const Ct &c = ct(ids[idx[c0 + b]]);
                    Ct o = new_ct(nq, 2, c.scale * t.scale);
                    o.slots = c.slots;
                    dst[b] = o.d;
                    outs[idx[c0 + b]] = put_ct(o);
                }
                scatter_words(dst, out, cts_);
                release(out);
            }
        }
    }

    void hybrid_fold(const std::vector<int> &ids, int rotations) {
        if (ids.empty() || rotations <= 0) return;
        std::map<int, std::vector<int>> bylevel;
        for (int id : ids) bylevel[ct(id).nq].push_back(id);
        for (auto &kv : bylevel) {
            const int nq = kv.first;
            const auto &v = kv.second;
            const size_t cts_ = (size_t)2 * nq * N;
            const int nb = (int)v.size();
            u64 *buf = alloc((size_t)nb * cts_), *rot = alloc((size_t)nb * cts_);
            std::vector<const Ct *> src(nb);
            std::vector<u64 *> dst(nb);
            for (int b = 0; b < nb; b++) {
                src[b] = &ct(v[b]);
                dst[b] = ct(v[b]).d;
            }
            gather_cts(buf, src, nq);
            for (int i = 1; i <= rotations; i++) {
                int k = slots >> i;
                u64 g = galois_of(k);
                u64 *key = rotation_key(g);
                rotate_batch(rot, buf, nq, nb, g, key, true);  // rot = buf + rot(buf)
                std::swap(buf, rot);
            }
            scatter_words(dst, buf, cts_);
            release(buf);
            release(rot);
        }
    }
};

static std::unique_ptr<Context> g_ctx;
static std::string g_err;

static Context &C() {
    if (!g_ctx) HB_THROW(HB_ESTATE, "B200 backend not initialised. Call NewScheme first.");
    return *g_ctx;
}

}  // namespace hb

using namespace hb;

#define HB_API extern "C" __attribute__((visibility("default")))

template <class F>
static int guard(F &&f) {
    try {
        f();
        return HB_OK;
    } catch (const HbError &e) {
        g_err = e.what();
        return e.code;
    } catch (const std::invalid_argument &e) {
        g_err = e.what();
        return HB_EINVAL;
    } catch (const std::out_of_range &e) {
        g_err = e.what();
        return HB_ENOENT;
    } catch (const std::bad_alloc &e) {
        g_err = "host allocation failed";
        return HB_ENOMEM;
    } catch (const std::exception &e) {
        g_err = e.what();
        return HB_ECUDA;
    }
}

#define OUT(p) \
    if (!(p)) HB_THROW(HB_EINVAL, "null output pointer")

HB_API const char *helrm_LastError(void) { return g_err.c_str(); }

HB_API int helrm_NewScheme(int logn, const int *logq, int nlogq, const int *logp, int nlogp, int logscale,
                           int hamming_weight, int dnum, uint64_t seed, int device) {
    return guard([&] {
        if (!logq || !logp || nlogq <= 0 || nlogp <= 0) HB_THROW(HB_EINVAL, "LogQ/LogP required");
        g_ctx.reset();
        auto c = std::make_unique<Context>();
        c->setup(logn, std::vector<int>(logq, logq + nlogq), std::vector<int>(logp, logp + nlogp), logscale,
                 hamming_weight, dnum, seed, device);
        g_ctx = std::move(c);
    });
}

HB_API int helrm_DeleteScheme(void) {
    return guard([&] { g_ctx.reset(); });
}

HB_API int helrm_GetModuliChain(uint64_t *out, int cap, int *n) {
    return guard([&] {
        Context &c = C();
        OUT(n);
        *n = c.L;
        for (int i = 0; i < c.L && i < cap; i++) out[i] = c.primes[i];
    });
}
HB_API int helrm_GetAuxModuliChain(uint64_t *out, int cap, int *n) {
    return guard([&] {
        Context &c = C();
        OUT(n);
        *n = c.K;
        for (int i = 0; i < c.K && i < cap; i++) out[i] = c.primes[c.L + i];
    });
}
HB_API int helrm_GetSchemeInfo(int *logn, int *slots, int *max_level, int *alpha, int *dnum) {
    return guard([&] {
        Context &c = C();
        if (logn) *logn = c.logN;
        if (slots) *slots = c.slots;
        if (max_level) *max_level = c.L - 1;
        if (alpha) *alpha = c.alpha;
        if (dnum) *dnum = c.dnum;
    });
}

HB_API int helrm_GenPrimes(int logn, const int *bits, int n, const uint64_t *used, int nused, uint64_t *out) {
    return guard([&] {
        if (!bits || !out || n < 0 || nused < 0 || (nused > 0 && !used)) HB_THROW(HB_EINVAL, "GenPrimes: bad arguments");
        std::vector<u64> u(used, used + nused);
        std::vector<u64> p = gen_primes(std::vector<int>(bits, bits + n), logn, u);
        for (int i = 0; i < n; i++) out[i] = p[i];
    });
}

HB_API int helrm_GenerateSecretKey(void) {
    return guard([&] { C().gen_secret(); });
}
HB_API int helrm_GeneratePublicKey(void) {
    return guard([&] { C().require_sk(); });
}
HB_API int helrm_GenerateRelinearizationKey(void) {
    return guard([&] {
        C().gen_relin();
        C().sync();
    });
}
HB_API int helrm_GenerateEvaluationKeys(void) {
    return guard([&] {
        Context &c = C();
        c.rotation_key(2ull * c.N - 1);
        c.sync();
    });
}
HB_API int helrm_AddRotationKey(int k) {
    return guard([&] {
        Context &c = C();
        u64 g = c.galois_of(k);
        if (g == 1) return;
        c.rotation_key(g);
        c.sync();
    });
}

HB_API int helrm_Encode(const double *values, int n, int level, double scale, int *out_pt) {
    return guard([&] {
        Context &c = C();
        OUT(out_pt);
        if (n < 0 || (n > 0 && !values)) HB_THROW(HB_EINVAL, "encode: bad values");
        std::vector<double> inter((size_t)2 * n);
        for (int i = 0; i < n; i++) {
            inter[2 * i] = values[i];
            inter[2 * i + 1] = 0.0;
        }
        *out_pt = c.encode(inter.data(), n, level, scale, false);
    });
}
HB_API int helrm_EncodeComplex(const double *inter, int n, int level, double scale, int *out_pt) {
    return guard([&] {
        Context &c = C();
        OUT(out_pt);
        if (n < 0 || (n > 0 && !inter)) HB_THROW(HB_EINVAL, "encode: bad values");
        *out_pt = c.encode(inter, n, level, scale, false);
    });
}
static void decode_impl(int pt, double *out, int cap, int *n, bool cplx) {
    Context &c = C();
    OUT(n);
    const Pt &p = c.pt(pt);
    std::vector<double> vals;
    c.decode_rows(p.d, p.nq, p.scale, vals);
    int cnt = std::min(cap, c.slots);
    if (cplx) {
        for (int i = 0; i < cnt; i++) {
            out[2 * i] = vals[2 * i];
            out[2 * i + 1] = vals[2 * i + 1];
        }
    } else {
        for (int i = 0; i < cnt; i++) out[i] = vals[2 * i];
    }
    *n = cnt;
}
HB_API int helrm_Decode(int pt, double *out, int cap, int *n) {
    return guard([&] { decode_impl(pt, out, cap, n, false); });
}
HB_API int helrm_DecodeComplex(int pt, double *out, int cap, int *n) {
    return guard([&] { decode_impl(pt, out, cap, n, true); });
}

HB_API int helrm_Encrypt(int pt, int *out_ct) {
    return guard([&] {
        Context &c = C();
        OUT(out_ct);
        const Pt &p = c.pt(pt);
        u64 ct_seed = hrand64(c.seed, 1000, c.enc_counter++);
        Ct o = c.encrypt_rows(p.d, p.nq, p.scale, ct_seed);
        o.slots = p.slots;
        *out_ct = c.put_ct(o);
    });
}
HB_API int helrm_EncryptSeeded(int pt, uint64_t seed, int *out_ct) {
    return guard([&] {
        Context &c = C();
        OUT(out_ct);
        const Pt &p = c.pt(pt);
        Ct o = c.encrypt_rows(p.d, p.nq, p.scale, seed);
        o.slots = p.slots;
        *out_ct = c.put_ct(o);
    });
}
HB_API int helrm_DropAx(int ct) {
    return guard([&] {
        Context &c = C();
        Ct &x = c.ct(ct);
        c.zero(x.d + (size_t)x.nq * c.N, (size_t)x.nq * c.N);
    });
}
HB_API int helrm_ExpandSeededAx(int ct, uint64_t seed) {
    return guard([&] {
        Context &c = C();
        Ct &x = c.ct(ct);
        sample_uniform(x.d + (size_t)x.nq * c.N, x.nq, nullptr, c.qmap(x.nq), seed, DOM_ENC_A, 0, 0, c.logN,
                       c.stream);
    });
}
HB_API int helrm_Decrypt(int ct, int *out_pt) {
    return guard([&] {
        Context &c = C();
        OUT(out_pt);
        c.require_sk();
        const Ct &x = c.ct(ct);
        const u64 *src = x.d;
        u64 *tmp = nullptr;
        if (x.npoly == 3) {
            if (!c.d_rlk) c.gen_relin();
            tmp = c.alloc((size_t)2 * x.nq * c.N);
            c.relinearize(tmp, x.d, x.nq);
            src = tmp;
        }
        Pt p;
        p.nq = x.nq;
        p.scale = x.scale;
        p.slots = x.slots;
        p.d = c.alloc((size_t)x.nq * c.N);
        ew_decrypt(p.d, src, c.d_sk, x.nq, c.logN, c.stream);
        if (tmp) c.release(tmp);
        *out_pt = c.put_pt(p);
    });
}

#define NEW_AND_INPLACE2(NAME, EXPR)                                           \
    HB_API int helrm_##NAME##New(int a, int b, int *out) {                     \
        return guard([&] {                                                     \
            Context &c = C();                                                  \
            OUT(out);                                                          \
            *out = (EXPR);                                                     \
        });                                                                    \
    }                                                                          \
    HB_API int helrm_##NAME(int a, int b) {                                    \
        return guard([&] {                                                     \
            Context &c = C();                                                  \
            int o = (EXPR);                                                    \
            c.replace_ct(a, o);                                                \
        });                                                                    \
    }

NEW_AND_INPLACE2(AddCiphertext, c.add_sub(a, b, false))
NEW_AND_INPLACE2(SubCiphertext, c.add_sub(a, b, true))
NEW_AND_INPLACE2(AddPlaintext, c.add_plain(a, b, false))
NEW_AND_INPLACE2(SubPlaintext, c.add_plain(a, b, true))
NEW_AND_INPLACE2(MulPlaintext, c.mul_plain(a, b))

static int mul_relin(Context &c, int a, int b) {
    if (!c.d_rlk) c.gen_relin();
    const Ct &ca = c.ct(a), &cb = c.ct(b);
    if (ca.npoly != 2 || cb.npoly != 2) HB_THROW(HB_ESTATE, "MulRelinCiphertext: operand is degree-2");
    int nq = std::min(ca.nq, cb.nq);
    Ct x = ca.nq == nq ? ca : c.drop_to(ca, nq);
    Ct y = cb.nq == nq ? cb : c.drop_to(cb, nq);
    u64 *t3 = c.alloc((size_t)3 * nq * c.N);
    ew_tensor(t3, x.d, y.d, nq, c.logN, c.stream);
    Ct o = c.new_ct(nq, 2, ca.scale * cb.scale);
    o.slots = std::max(ca.slots, cb.slots);
    c.relinearize(o.d, t3, nq);
    c.release(t3);
    if (x.d != ca.d) c.release(x.d);
    if (y.d != cb.d) c.release(y.d);
    return c.put_ct(o);
}
NEW_AND_INPLACE2(MulRelinCiphertext, mul_relin(c, a, b))

// the pairs of one level (the lower of the two operands') gathered into one
// batch: one batched tensor product and one batched relinearisation, the
// same arithmetic as mul_relin per pair
HB_API int helrm_MulRelinCiphertextBatchNew(const int *a, const int *b, int n, int *out) {
    return guard([&] {
        Context &c = C();
        if (n < 0 || (n > 0 && (!a || !b || !out))) HB_THROW(HB_EINVAL, "MulRelinCiphertextBatchNew: bad arguments");
        if (!c.d_rlk) c.gen_relin();
        std::map<int, std::vector<int>> groups;
        for (int i = 0; i < n; i++) {
            const Ct &ca = c.ct(a[i]), &cb = c.ct(b[i]);
            if (ca.npoly != 2 || cb.npoly != 2) HB_THROW(HB_ESTATE, "MulRelinCiphertext: operand is degree-2");
            groups[std::min(ca.nq, cb.nq)].push_back(i);
        }
        for (auto &kv : groups) {
            const int nq = kv.first;
            const auto &idx = kv.second;
            const int nb = (int)idx.size();
            const size_t w2 = (size_t)2 * nq * c.N;
            std::vector<const Ct *> va(nb), vb(nb);
            for (int k = 0; k < nb; k++) {
                va[k] = &c.ct(a[idx[k]]);
                vb[k] = &c.ct(b[idx[k]]);
            }
            u64 *A = c.alloc((size_t)nb * w2), *B = c.alloc((size_t)nb * w2);
            c.gather_cts(A, va, nq);  // the first nq rows of each polynomial
            c.gather_cts(B, vb, nq);
            u64 *t3 = c.alloc((size_t)nb * 3 * nq * c.N);
            ew_tensor_batch(t3, A, B, nq, nq, nq, nb, w2, w2, c.logN, c.stream);
            c.release(A);
            c.release(B);
            u64 *R = c.alloc((size_t)nb * w2);
            c.relinearize_batch(R, t3, nq, nb);
            c.release(t3);
            std::vector<u64 *> dst(nb);
            std::vector<int> fresh(nb);
            for (int k = 0; k < nb; k++) {
                const Ct &ca = *va[k], &cb = *vb[k];
                Ct o = c.new_ct(nq, 2, ca.scale * cb.scale);
                o.slots = std::max(ca.slots, cb.slots);
                dst[k] = o.d;
                fresh[k] = c.put_ct(o);
            }
            c.scatter_words(dst, R, w2);
            c.release(R);
            for (int k = 0; k < nb; k++) out[idx[k]] = fresh[k];
        }
    });
}

// ---- polynomial evaluation ----------------------------------------------------
static PolyPlan &poly_plan(Context &c, bool cheb, int nq0, double s1, const std::vector<double> &co, double S) {
    std::string key;
    auto put = [&](const void *p, size_t n) { key.append((const char *)p, n); };
    const int b = cheb ? 1 : 0;
    put(&b, sizeof b);
    put(&nq0, sizeof nq0);
    put(&s1, sizeof s1);
    put(&S, sizeof S);
    put(co.data(), co.size() * sizeof(double));
    auto it = c.poly_plans.find(key);
    if (it != c.poly_plans.end()) return it->second;
    if (c.poly_plans.size() >= 64) {
        for (auto &kv : c.poly_plans) c.release(kv.second.d_consts);
        c.poly_plans.clear();
    }
    PolyPlan pl = plan_polynomial(c.primes, cheb, nq0, s1, co, S);
    pl.d_consts = c.alloc(pl.consts.size());
    cuda_check(cudaMemcpyAsync(pl.d_consts, pl.consts.data(), pl.consts.size() * 8, cudaMemcpyHostToDevice, c.stream),
               "polynomial constants");
    c.sync();
    return c.poly_plans.emplace(key, std::move(pl)).first->second;
}

// replay a plan over nb ciphertexts of the plan's input rows and scale
static std::vector<int> poly_run(Context &c, const PolyPlan &pl, const std::vector<int> &ids) {
    const int nb = (int)ids.size();
    const size_t N = c.N;
    const size_t nv = pl.vnq.size();
    std::vector<u64 *> vd(nv, nullptr);
    std::vector<char> own(nv, 1);
    auto stride = [&](int v) { return (size_t)2 * pl.vnq[v] * N; };
    if (nb == 1) {
        vd[0] = c.ct(ids[0]).d;
        own[0] = 0;
    } else {
        std::vector<const Ct *> v;
        for (int id : ids) v.push_back(&c.ct(id));
        vd[0] = c.alloc((size_t)nb * stride(0));
        c.gather_cts(vd[0], v, pl.vnq[0]);
    }
    for (size_t i = 0; i < pl.ops.size(); i++) {
        const PolyOp &o = pl.ops[i];
        const int nq = pl.vnq[o.out];
        vd[o.out] = c.alloc((size_t)nb * stride(o.out));
        if (o.kind == PO_MUL) {
            u64 *t3 = c.alloc((size_t)nb * 3 * nq * N);
            ew_tensor_batch(t3, vd[o.a], vd[o.b], nq, pl.vnq[o.a], pl.vnq[o.b], nb, stride(o.a), stride(o.b), c.logN,
                            c.stream);
            c.relinearize_batch(vd[o.out], t3, nq, nb);
            c.release(t3);
        } else if (o.kind == PO_LIN) {
            LinCombArgs a{};
            a.n = o.nt;
            for (int t = 0; t < o.nt; t++) {
                const int v = pl.terms[o.t0 + t];
                a.x[t] = vd[v];
                a.xs[t] = stride(v);
                a.nq[t] = pl.vnq[v];
            }
            a.coef = pl.d_consts + o.coef;
            a.k0 = o.k0 >= 0 ? pl.d_consts + o.k0 : nullptr;
            ew_lincomb(vd[o.out], a, nq, nb, stride(o.out), c.logN, c.stream);
        } else if (o.kind == PO_RESCALE) {
            c.rescale(vd[o.out], vd[o.a], 2, pl.vnq[o.a], nb, stride(o.a), stride(o.out));
        } else {
            ew_add(vd[o.out], vd[o.a], vd[o.b], nb * 2 * nq, c.qmap(nq), c.logN, c.stream);
        }
        auto drop = [&](int v) {
            if (v >= 0 && v != pl.out && own[v] && vd[v] && pl.last_use[v] == (int)i) {
                c.release(vd[v]);
                vd[v] = nullptr;
            }
        };
        drop(o.a);
        drop(o.b);
        for (int t = 0; t < o.nt; t++) drop(pl.terms[o.t0 + t]);
    }
    std::vector<int> outs;
    const int onq = pl.vnq[pl.out];
    if (nb == 1) {
        Ct o;
        o.d = vd[pl.out];
        o.nq = onq;
        o.npoly = 2;
        o.scale = pl.target;
        o.slots = c.ct(ids[0]).slots;
        outs.push_back(c.put_ct(o));
    } else {
        std::vector<u64 *> dsts;
        for (int id : ids) {
            Ct o = c.new_ct(onq, 2, pl.target);
            o.slots = c.ct(id).slots;
            dsts.push_back(o.d);
            outs.push_back(c.put_ct(o));
        }
        c.scatter_words(dsts, vd[pl.out], stride(pl.out));
        c.release(vd[pl.out]);
    }
    return outs;
}

// ciphertexts grouped by (rows, scale), one plan replay per group
static void eval_polynomial(Context &c, const int *ids, int nb, const double *coeffs, int n, int cheb, double S,
                            int *outs) {
    if (nb <= 0 || !ids || !outs) HB_THROW(HB_EINVAL, "EvaluatePolynomial: empty input");
    if (n < 3 || !coeffs) HB_THROW(HB_EINVAL, "EvaluatePolynomial: the native evaluation needs degree >= 2");
    if (!(S > 0)) HB_THROW(HB_EINVAL, "EvaluatePolynomial: output scale must be positive");
    const std::vector<double> co(coeffs, coeffs + n);
    for (double v : co)
        if (!std::isfinite(v)) HB_THROW(HB_EINVAL, "EvaluatePolynomial: non-finite coefficient");
    if (!c.d_rlk) c.gen_relin();
    std::map<std::pair<int, double>, std::vector<int>> groups;
    for (int i = 0; i < nb; i++) {
        const Ct &x = c.ct(ids[i]);
        if (x.npoly != 2)
            HB_THROW(HB_ESTATE, "EvaluatePolynomial: relinearize before evaluating a polynomial.");
        groups[{x.nq, x.scale}].push_back(i);
    }
    for (auto &kv : groups) {
        const PolyPlan &pl = poly_plan(c, cheb != 0, kv.first.first, kv.first.second, co, S);
        std::vector<int> g;
        for (int i : kv.second) g.push_back(ids[i]);
        const std::vector<int> r = poly_run(c, pl, g);
        for (size_t j = 0; j < r.size(); j++) outs[kv.second[j]] = r[j];
    }
}

HB_API int helrm_EvaluatePolynomial(int ct, const double *coeffs, int n, int chebyshev, double scale, int *out) {
    return guard([&] {
        Context &c = C();
        OUT(out);
        eval_polynomial(c, &ct, 1, coeffs, n, chebyshev, scale, out);
    });
}

HB_API int helrm_EvaluatePolynomialBatch(const int *cts, int nb, const double *coeffs, int n, int chebyshev,
                                         double scale, int *outs) {
    return guard([&] {
        Context &c = C();
        eval_polynomial(c, cts, nb, coeffs, n, chebyshev, scale, outs);
    });
}

HB_API int helrm_PolynomialPlanInfo(int nq, double in_scale, const double *coeffs, int n, int chebyshev, double scale,
                                    int *info) {
    return guard([&] {
        Context &c = C();
        if (!info || !coeffs || nq < 1 || nq > c.L) HB_THROW(HB_EINVAL, "PolynomialPlanInfo: bad arguments");
        const PolyPlan pl =
            plan_polynomial(c.primes, chebyshev != 0, nq, in_scale, std::vector<double>(coeffs, coeffs + n), scale);
        info[0] = pl.depth;
        info[1] = pl.products;
        info[2] = pl.rescales;
        info[3] = pl.bs;
    });
}

// a fresh ciphertext -ct, the input untouched, as every reference backend
// returns it (lattigo evaluator.go:68-78, cheddar_pybind.cu:1798-1803)
HB_API int helrm_Negate(int ct, int *out) {
    return guard([&] {
        Context &c = C();
        OUT(out);
        const Ct &x = c.ct(ct);
        Ct o = c.new_ct(x.nq, x.npoly, x.scale);
        o.slots = x.slots;
        ew_neg(o.d, x.d, x.npoly * x.nq, c.qmap(x.nq), c.logN, c.stream);
        *out = c.put_ct(o);
    });
}

HB_API int helrm_MulPlaintextAccumNew(const int *cts, const int *pts, int n, int *out) {
    return guard([&] {
        Context &c = C();
        OUT(out);
        if (n <= 0 || !cts || !pts) HB_THROW(HB_EINVAL, "MulPlaintextAccumNew: empty input");
        *out = c.mac(std::vector<int>(cts, cts + n), std::vector<int>(pts, pts + n));
    });
}

#define SCALAR_OPS(NAME, KIND, T)                                              \
    HB_API int helrm_##NAME##New(int ct, T s, int *out) {                      \
        return guard([&] {                                                     \
            Context &c = C();                                                  \
            OUT(out);                                                          \
            *out = c.scalar_op(ct, (long double)s, KIND);                      \
        });                                                                    \
    }                                                                          \
    HB_API int helrm_##NAME(int ct, T s) {                                     \
        return guard([&] {                                                     \
            Context &c = C();                                                  \
            int o = c.scalar_op(ct, (long double)s, KIND);                     \
            c.replace_ct(ct, o);                                               \
        });                                                                    \
    }
SCALAR_OPS(AddScalar, 0, double)
SCALAR_OPS(SubScalar, 1, double)
SCALAR_OPS(MulScalarInt, 2, int64_t)
SCALAR_OPS(MulScalarFloat, 3, double)

static int rescale_new(Context &c, int id) {
    const Ct &x = c.ct(id);
    if (x.nq < 2) HB_THROW(HB_ESTATE, "RescaleNew: ciphertext already at level 0.");
    Ct o = c.new_ct(x.nq - 1, x.npoly, x.scale / (double)c.primes[x.nq - 1]);
    o.slots = x.slots;
    c.rescale(o.d, x.d, x.npoly, x.nq, 1, 0, 0);
    return c.put_ct(o);
}
HB_API int helrm_RescaleNew(int ct, int *out) {
    return guard([&] {
        Context &c = C();
        OUT(out);
        *out = rescale_new(c, ct);
    });
}
HB_API int helrm_Rescale(int ct) {
    return guard([&] {
        Context &c = C();
        int o = rescale_new(c, ct);
        c.replace_ct(ct, o);
    });
}
HB_API int helrm_RescaleBatch(const int *cts, int n) {
    return guard([&] {
        Context &c = C();
        if (n < 0 || (n > 0 && !cts)) HB_THROW(HB_EINVAL, "RescaleBatch: bad arguments");
        // ciphertexts of the same level and degree are rescaled together:
        // gathered into one batch, rescaled with batched kernels, scattered
        // into fresh ciphertexts that replace the inputs (same ids)
        std::map<std::pair<int, int>, std::vector<int>> groups;
        for (int i = 0; i < n; i++) {
            const Ct &x = c.ct(cts[i]);
            if (x.nq < 2) HB_THROW(HB_ESTATE, "RescaleBatch: ciphertext already at level 0.");
            groups[{x.nq, x.npoly}].push_back(cts[i]);
        }
        for (auto &kv : groups) {
            const int nq = kv.first.first, npoly = kv.first.second;
            const auto &v = kv.second;
            const int nb = (int)v.size();
            if (npoly != 2) {
                for (int id : v) c.replace_ct(id, rescale_new(c, id));
                continue;
            }
            const size_t in_w = (size_t)2 * nq * c.N, out_w = (size_t)2 * (nq - 1) * c.N;
            u64 *in = c.alloc((size_t)nb * in_w), *out = c.alloc((size_t)nb * out_w);
            std::vector<const Ct *> src(nb);
            for (int b = 0; b < nb; b++) src[b] = &c.ct(v[b]);
            c.gather_cts(in, src, nq);
            c.rescale(out, in, 2, nq, nb, in_w, out_w);
            std::vector<u64 *> dst(nb);
            std::vector<int> fresh(nb);
            for (int b = 0; b < nb; b++) {
                const Ct &x = c.ct(v[b]);
                Ct o = c.new_ct(nq - 1, 2, x.scale / (double)c.primes[nq - 1]);
                o.slots = x.slots;
                dst[b] = o.d;
                fresh[b] = c.put_ct(o);
            }
            c.scatter_words(dst, out, out_w);
            c.release(in);
            c.release(out);
            for (int b = 0; b < nb; b++) c.replace_ct(v[b], fresh[b]);
        }
    });
}

HB_API int helrm_AlignToLevelNew(int ct, int level, int *out) {
    return guard([&] {
        Context &c = C();
        OUT(out);
        const Ct &x = c.ct(ct);
        if (x.nq - 1 < level)
            HB_THROW(HB_ESTATE, "AlignToLevelNew: input level " + std::to_string(x.nq - 1) + " below target " +
                                    std::to_string(level) + ".");
        if (level < 0) HB_THROW(HB_EINVAL, "AlignToLevelNew: negative level");
        *out = c.put_ct(c.drop_to(x, level + 1));
    });
}

static int rotate_new(Context &c, int id, int k) {
    const Ct &x = c.ct(id);
    if (x.npoly != 2) HB_THROW(HB_ESTATE, "RotateNew: input is degree-2; relinearize first.");
    u64 g = c.galois_of(k);
    if (g == 1) return c.put_ct(c.drop_to(x, x.nq));
    u64 *key = c.rotation_key(g);
    Ct o = c.new_ct(x.nq, 2, x.scale);
    o.slots = x.slots;
    c.rotate_batch(o.d, x.d, x.nq, 1, g, key);
    return c.put_ct(o);
}
HB_API int helrm_RotateNew(int ct, int k, int *out) {
    return guard([&] {
        Context &c = C();
        OUT(out);
        *out = rotate_new(c, ct, k);
    });
}
HB_API int helrm_Rotate(int ct, int k) {
    return guard([&] {
        Context &c = C();
        int o = rotate_new(c, ct, k);
        c.replace_ct(ct, o);
    });
}
static int conj_new(Context &c, int id) {
    const Ct &x = c.ct(id);
    if (x.npoly != 2) HB_THROW(HB_ESTATE, "ConjugateNew: input is degree-2; relinearize first.");
    u64 g = 2ull * c.N - 1;
    u64 *key = c.rotation_key(g);
    Ct o = c.new_ct(x.nq, 2, x.scale);
    o.slots = x.slots;
    c.rotate_batch(o.d, x.d, x.nq, 1, g, key);
    return c.put_ct(o);
}
// slot-wise multiplication by sqrt(-1): key-free, no level
// (cheddar_pybind.cu:1825-1837, bindings.py:607-612)
static int mul_iunit_new(Context &c, int id) {
    const Ct &x = c.ct(id);
    Ct o = c.new_ct(x.nq, x.npoly, x.scale);
    o.slots = x.slots;
    ew_mul_iunit(o.d, x.d, x.npoly * x.nq, x.nq, c.d_iunit, c.logN, c.stream);
    return c.put_ct(o);
}
HB_API int helrm_MulImaginaryUnitNew(int ct, int *out) {
    return guard([&] {
        Context &c = C();
        OUT(out);
        *out = mul_iunit_new(c, ct);
    });
}
HB_API int helrm_MulImaginaryUnit(int ct) {
    return guard([&] {
        Context &c = C();
        int o = mul_iunit_new(c, ct);
        c.replace_ct(ct, o);
    });
}

// the server side of complex-lane packing (orion/core/lane_packing.py:84-115):
// packed p = (x + i y) / 2 -> x = p + conj(p), y = -i (p - conj(p)); one
// batched conjugation key switch for all packed ciphertexts, both lanes in
// one pass.  outs[2m], outs[2m+1] are the lanes of packed[m]; the first
// num_real are kept (an odd count drops the last zero-padded partner).
static void unpack_lanes(Context &c, const int *ids, int n, int num_real, int *outs) {
    if (n <= 0 || !ids || !outs || num_real < 0 || num_real > 2 * n)
        HB_THROW(HB_EINVAL, "UnpackLanes: bad arguments");
    const Ct &x0 = c.ct(ids[0]);
    const int nq = x0.nq;
    for (int i = 0; i < n; i++) {
        const Ct &x = c.ct(ids[i]);
        if (x.npoly != 2) HB_THROW(HB_ESTATE, "UnpackLanes: input is degree-2; relinearize first.");
        if (x.nq != nq) HB_THROW(HB_ESTATE, "UnpackLanes: packed ciphertexts must share one level");
    }
    const u64 g = 2ull * c.N - 1;
    u64 *key = c.rotation_key(g);
    const size_t words = (size_t)2 * nq * c.N;
    const int chunk = std::min(n, 64);
    u64 *buf = c.alloc((size_t)chunk * words), *cj = c.alloc((size_t)chunk * words);
    for (int c0 = 0; c0 < n; c0 += chunk) {
        const int cnt = std::min(chunk, n - c0);
        std::vector<const Ct *> v;
        for (int i = 0; i < cnt; i++) v.push_back(&c.ct(ids[c0 + i]));
        c.gather_cts(buf, v, nq);
        c.rotate_batch(cj, buf, nq, cnt, g, key);
        PtrBatchW ev{}, od{};
        std::vector<Ct> made;
        for (int i = 0; i < cnt; i++) {
            const Ct &x = c.ct(ids[c0 + i]);
            for (int lane = 0; lane < 2; lane++) {
                Ct o = c.new_ct(nq, 2, x.scale);
                o.slots = x.slots;
                (lane ? od : ev).p[i] = o.d;
                made.push_back(o);
            }
        }
        lane_split(ev, od, buf, cj, nq, cnt, c.d_iunit, c.logN, c.stream);
        for (int i = 0; i < cnt; i++)
            for (int lane = 0; lane < 2; lane++) {
                const int r = 2 * (c0 + i) + lane;
                Ct &o = made[(size_t)2 * i + lane];
                if (r < num_real)
                    outs[r] = c.put_ct(o);
                else
                    c.release(o.d);
            }
    }
    c.release(buf);
    c.release(cj);
}
HB_API int helrm_UnpackLanes(const int *packed, int n, int num_real, int *outs) {
    return guard([&] {
        Context &c = C();
        unpack_lanes(c, packed, n, num_real, outs);
    });
}

HB_API int helrm_EncodeBatch(const double *values, int count, int n, int level, double scale, int *outs) {
    return guard([&] {
        Context &c = C();
        if (count <= 0 || !outs || n < 0 || (n > 0 && !values)) HB_THROW(HB_EINVAL, "EncodeBatch: bad arguments");
        if (level < 0 || level >= c.L) HB_THROW(HB_EINVAL, "encode: level out of range");
        if (!(scale > 0)) scale = c.default_scale;
        std::vector<u64 *> d;
        std::vector<Pt> made;
        for (int i = 0; i < count; i++) {
            Pt p;
            p.nq = level + 1;
            p.ext = false;
            p.scale = scale;
            p.slots = c.slots;
            p.d = c.alloc((size_t)p.nq * c.N);
            d.push_back(p.d);
            made.push_back(p);
        }
        c.encode_device(values, n, false, count, level + 1, false, scale, d.data());
        for (int i = 0; i < count; i++) outs[i] = c.put_pt(made[i]);
    });
}

HB_API int helrm_ModRaiseNew(int ct, int *out) {
    return guard([&] {
        Context &c = C();
        OUT(out);
        *out = c.mod_raise(ct);
    });
}

HB_API int helrm_ConjugateNew(int ct, int *out) {
    return guard([&] {
        Context &c = C();
        OUT(out);
        *out = conj_new(c, ct);
    });
}
HB_API int helrm_Conjugate(int ct) {
    return guard([&] {
        Context &c = C();
        int o = conj_new(c, ct);
        c.replace_ct(ct, o);
    });
}

HB_API int helrm_RotateBatchNew(int ct, const int *ks, int n, int *outs) {
    return guard([&] {
        Context &c = C();
        if (n <= 0) return;
        if (!ks || !outs) HB_THROW(HB_EINVAL, "RotateBatchNew: null array");
        const Ct &x = c.ct(ct);
        if (x.npoly != 2) HB_THROW(HB_ESTATE, "RotateBatchNew: input is degree-2; relinearize first.");
        std::vector<u64> gs;
        std::vector<int> pos;
        std::vector<u64 *> bufs;
        std::vector<int> ids(n, 0);
        for (int i = 0; i < n; i++) {
            u64 g = c.galois_of(ks[i]);
            if (g == 1) {
                ids[i] = c.put_ct(c.drop_to(x, x.nq));
                continue;
            }
            Ct o = c.new_ct(x.nq, 2, x.scale);
            o.slots = x.slots;
            ids[i] = c.put_ct(o);
            gs.push_back(g);
            bufs.push_back(o.d);
        }
        if (!gs.empty()) c.rotate_hoisted(x.d, x.nq, 1, gs, bufs, 0);
        for (int i = 0; i < n; i++) outs[i] = ids[i];
    });
}

HB_API int helrm_GenerateLinearTransform(const int *diag_idxs, int n, const double *data, int width, int level,
                                         double bsgs_ratio, int *out_lt) {
    return guard([&] {
        Context &c = C();
        OUT(out_lt);
        if (!diag_idxs || !data) HB_THROW(HB_EINVAL, "GenerateLinearTransform: null input");
        *out_lt = c.generate_lt(diag_idxs, n, data, width, level, bsgs_ratio);
    });
}
// complex diagonals (interleaved re, im when cplx != 0) encoded at an
// explicit plaintext scale (<= 0: the default scale)
HB_API int helrm_GenerateLinearTransformEx(const int *diag_idxs, int n, const double *data, int width, int level,
                                           double bsgs_ratio, int cplx, double scale, int *out_lt) {
    return guard([&] {
        Context &c = C();
        OUT(out_lt);
        if (!diag_idxs || !data) HB_THROW(HB_EINVAL, "GenerateLinearTransform: null input");
        *out_lt = c.generate_lt(diag_idxs, n, data, width, level, bsgs_ratio, cplx != 0, scale);
    });
}
HB_API int helrm_EvaluateLinearTransformBatch(int lt, const int *cts, int n, int *outs) {
    return guard([&] {
        Context &c = C();
        if (n <= 0) return;
        if (!cts || !outs) HB_THROW(HB_EINVAL, "EvaluateLinearTransformBatch: null array");
        std::vector<int> o;
        c.eval_lt_batch(lt, std::vector<int>(cts, cts + n), o);
        for (int i = 0; i < n; i++) outs[i] = o[i];
    });
}
HB_API int helrm_EvaluateLinearTransform(int lt, int ct, int *out) {
    return helrm_EvaluateLinearTransformBatch(lt, &ct, 1, out);
}
HB_API int helrm_DeleteLinearTransform(int lt) {
    return guard([&] {
        Context &c = C();
        auto it = c.lts.find(lt);
        if (it == c.lts.end()) return;
        c.sync();
        c.free_lt(*it->second);
        c.lts.erase(it);
    });
}
HB_API int helrm_GetLinearTransformRotationKeys(int lt, int *out, int cap, int *n) {
    return guard([&] {
        Context &c = C();
        OUT(n);
        auto v = c.lt_rotation_keys(c.lt(lt));
        *n = (int)v.size();
        for (int i = 0; i < (int)v.size() && i < cap; i++) out[i] = v[i];
    });
}
HB_API int helrm_GetLinearTransformInfo(int lt, int *bs, int *ndiag, int *ngiant, int *level) {
    return guard([&] {
        Context &c = C();
        LinTrans &t = c.lt(lt);
        if (bs) *bs = t.use_bsgs ? t.bs : 0;
        if (ndiag) *ndiag = (int)t.ks.size();
        if (ngiant) *ngiant = (int)t.groups.size();
        if (level) *level = t.level;
    });
}
HB_API int helrm_HybridFoldBatch(const int *cts, int n, int rotations) {
    return guard([&] {
        Context &c = C();
        if (n <= 0) return;
        c.hybrid_fold(std::vector<int>(cts, cts + n), rotations);
    });
}

HB_API int helrm_EncodeConstantNew(double scalar, int level, double scale, int *out) {
    return guard([&] {
        OUT(out);
        *out = C().encode_constant(scalar, level, scale);
    });
}
HB_API int helrm_DeleteConstant(int id) {
    return guard([&] {
        Context &c = C();
        c.konst(id);
        c.konsts.erase(id);
    });
}
HB_API int helrm_MulConstantAccumNew(const int *cts, const int *consts, int n, int *out) {
    return guard([&] {
        Context &c = C();
        OUT(out);
        if (!cts || !consts || n <= 0) HB_THROW(HB_EINVAL, "MulConstantAccumNew: bad arguments");
        const int t = c.pack_constant_table(consts, n, 1);
        try {
            *out = c.table_matmul_ids(cts, n, c.table(t))[0];
        } catch (...) {
            c.delete_table(t);
            throw;
        }
        c.delete_table(t);
    });
}
HB_API int helrm_PackConstantTableNew(const int *consts, int n, int rows, int *out) {
    return guard([&] {
        OUT(out);
        if (!consts) HB_THROW(HB_EINVAL, "PackConstantTableNew: null ids");
        *out = C().pack_constant_table(consts, n, rows);
    });
}
HB_API int helrm_PackPlaintextTableNew(const int *pts, int n, int rows, int *out) {
    return guard([&] {
        OUT(out);
        if (!pts) HB_THROW(HB_EINVAL, "PackPlaintextTableNew: null ids");
        *out = C().pack_plaintext_table(pts, n, rows);
    });
}
HB_API int helrm_DeleteTable(int table) {
    return guard([&] { C().delete_table(table); });
}
HB_API int helrm_GetTableShape(int table, int *rows, int *cols, int *level) {
    return guard([&] {
        Context::Table &t = C().table(table);
        if (rows) *rows = t.rows;
        if (cols) *cols = t.cols;
        if (level) *level = t.level;
    });
}
HB_API int helrm_MulTableMatMulNew(const int *cts, int n, int table, int *outs) {
    return guard([&] {
        Context &c = C();
        OUT(outs);
        if (!cts) HB_THROW(HB_EINVAL, "MulTableMatMulNew: null ids");
        std::vector<int> o = c.table_matmul_ids(cts, n, c.table(table));
        for (size_t i = 0; i < o.size(); i++) outs[i] = o[i];
    });
}
HB_API int helrm_DeleteCiphertext(int ct) {
    return guard([&] {
        if (g_ctx) g_ctx->del_ct(ct);
    });
}
HB_API int helrm_DeletePlaintext(int pt) {
    return guard([&] {
        if (g_ctx) g_ctx->del_pt(pt);
    });
}
HB_API int helrm_GetCiphertextLevel(int ct, int *level) {
    return guard([&] {
        OUT(level);
        *level = C().ct(ct).nq - 1;
    });
}
HB_API int helrm_GetPlaintextLevel(int pt, int *level) {
    return guard([&] {
        OUT(level);
        *level = C().pt(pt).nq - 1;
    });
}
HB_API int helrm_GetCiphertextScale(int ct, double *scale) {
    return guard([&] {
        OUT(scale);
        *scale = C().ct(ct).scale;
    });
}
HB_API int helrm_GetPlaintextScale(int pt, double *scale) {
    return guard([&] {
        OUT(scale);
        *scale = C().pt(pt).scale;
    });
}
HB_API int helrm_SetCiphertextScale(int ct, double scale) {
    return guard([&] { C().ct(ct).scale = scale; });
}
HB_API int helrm_SetPlaintextScale(int pt, double scale) {
    return guard([&] { C().pt(pt).scale = scale; });
}
HB_API int helrm_GetCiphertextSlots(int ct, int *s) {
    return guard([&] {
        OUT(s);
        *s = C().ct(ct).slots;
    });
}
HB_API int helrm_GetPlaintextSlots(int pt, int *s) {
    return guard([&] {
        OUT(s);
        *s = C().pt(pt).slots;
    });
}
HB_API int helrm_SetCiphertextSlots(int ct, int slots) {
    return guard([&] {
        Context &c = C();
        Ct &x = c.ct(ct);
        if (slots <= 0 || slots > x.slots || x.slots % slots != 0)
            HB_THROW(HB_EINVAL, "SetCiphertextSlots: narrowing retag only (divisor of the current width)");
        x.slots = slots;
    });
}
HB_API int helrm_GetCiphertextDegree(int ct, int *d) {
    return guard([&] {
        OUT(d);
        *d = C().ct(ct).npoly - 1;
    });
}
HB_API int helrm_GetLiveCounts(int *cts, int *pts) {
    return guard([&] {
        Context &c = C();
        if (cts) *cts = (int)c.cts.size();
        if (pts) *pts = (int)c.pts.size();
    });
}
HB_API int helrm_GetCiphertextBytes(int ct, double *bytes) {
    return guard([&] {
        Context &c = C();
        OUT(bytes);
        const Ct &x = c.ct(ct);
        *bytes = (double)x.npoly * x.nq * c.N * 8;
    });
}
HB_API int helrm_GetMemoryMB(double *live, double *peak, double *keys) {
    return guard([&] {
        Context &c = C();
        if (live) *live = c.live / 1048576.0;
        if (peak) *peak = c.peak / 1048576.0;
        if (keys) *keys = c.key_bytes / 1048576.0;
    });
}

HB_API int helrm_GetCiphertextData(int ct, uint64_t *out, size_t words) {
    return guard([&] {
        Context &c = C();
        const Ct &x = c.ct(ct);
        size_t need = (size_t)x.npoly * x.nq * c.N;
        if (!out || words < need) HB_THROW(HB_EINVAL, "GetCiphertextData: buffer too small");
        cuda_check(cudaMemcpyAsync(out, x.d, need * 8, cudaMemcpyDeviceToHost, c.stream), "d2h");
        c.sync();
    });
}
HB_API int helrm_NewCiphertextFromData(const uint64_t *data, int level, int npoly, double scale, int *out) {
    return guard([&] {
        Context &c = C();
        OUT(out);
        if (level < 0 || level >= c.L || npoly < 2 || npoly > 3 || !data)
            HB_THROW(HB_EINVAL, "NewCiphertextFromData: bad level/degree");
        Ct o = c.new_ct(level + 1, npoly, scale);
        cuda_check(cudaMemcpyAsync(o.d, data, (size_t)npoly * (level + 1) * c.N * 8, cudaMemcpyHostToDevice,
                                   c.stream),
                   "h2d");
        c.sync();
        *out = c.put_ct(o);
    });
}
HB_API int helrm_UploadCiphertextsAsync(const uint64_t *const *host, int n, int level, int npoly, double scale,
                                        int *out_ids) {
    return guard([&] {
        Context &c = C();
        if (!host || !out_ids || n <= 0 || level < 0 || level >= c.L || npoly < 2 || npoly > 3)
            HB_THROW(HB_EINVAL, "UploadCiphertextsAsync: bad arguments");
        for (int i = 0; i < n; i++)
            if (!host[i]) HB_THROW(HB_EINVAL, "UploadCiphertextsAsync: null host buffer");
        c.ensure_xfer();
        const size_t words = (size_t)npoly * (level + 1) * c.N;
        for (int i = 0; i < n; i++) {
            Ct o;
            o.nq = level + 1;
            o.npoly = npoly;
            o.scale = scale;
            o.slots = c.slots;
            o.d = c.alloc_on(words, c.up);
            cuda_check(cudaMemcpyAsync(o.d, host[i], words * 8, cudaMemcpyHostToDevice, c.up), "h2d");
            out_ids[i] = c.put_ct(o);
        }
        c.wait_for(c.stream, c.up, c.ev_up);
    });
}
HB_API int helrm_DownloadCiphertextsAsync(const int *ids, int n, uint64_t *const *host, size_t words_each) {
    return guard([&] {
        Context &c = C();
        if (!ids || !host || n <= 0) HB_THROW(HB_EINVAL, "DownloadCiphertextsAsync: bad arguments");
        for (int i = 0; i < n; i++) {
            const Ct &x = c.ct(ids[i]);
            if (!host[i] || words_each < (size_t)x.npoly * x.nq * c.N)
                HB_THROW(HB_EINVAL, "DownloadCiphertextsAsync: buffer too small");
        }
        c.ensure_xfer();
        c.wait_for(c.dn, c.stream, c.ev_comp);
        for (int i = 0; i < n; i++) {
            Ct &x = c.ct(ids[i]);
            cuda_check(cudaMemcpyAsync(host[i], x.d, (size_t)x.npoly * x.nq * c.N * 8, cudaMemcpyDeviceToHost, c.dn),
                       "d2h");
            x.xfer = true;
        }
    });
}
HB_API int helrm_CiphertextsToDevice(const int *ids, int n, uint64_t *d_out, size_t words_each) {
    return guard([&] {
        Context &c = C();
        if (!ids || !d_out || n <= 0) HB_THROW(HB_EINVAL, "CiphertextsToDevice: bad arguments");
        for (int i = 0; i < n; i++) {
            const Ct &x = c.ct(ids[i]);
            const size_t words = (size_t)x.npoly * x.nq * c.N;
            if (words > words_each) HB_THROW(HB_EINVAL, "CiphertextsToDevice: item smaller than the ciphertext");
            cuda_check(cudaMemcpyAsync(d_out + (size_t)i * words_each, x.d, words * 8, cudaMemcpyDeviceToDevice,
                                       c.stream),
                       "CiphertextsToDevice");
        }
        c.sync();  // the caller's stream (a collective) reads the buffer next
    });
}
HB_API int helrm_NewCiphertextsFromDeviceSum(const uint64_t *d_in, int n, int level, int npoly, double scale,
                                             int *out_ids) {
    return guard([&] {
        Context &c = C();
        if (!d_in || !out_ids || n <= 0 || level < 0 || level >= c.L || npoly < 1 || npoly > 3)
            HB_THROW(HB_EINVAL, "NewCiphertextsFromDeviceSum: bad arguments");
        const int nq = level + 1;
        const size_t words = (size_t)npoly * nq * c.N;
        for (int i = 0; i < n; i++) {
            Ct o = c.new_ct(nq, npoly, scale);
            o.slots = c.slots;
            ew_reduce_rows(o.d, (const u64 *)d_in + (size_t)i * words, npoly * nq, c.qmap(nq), c.logN, c.stream);
            out_ids[i] = c.put_ct(o);
        }
    });
}
HB_API int helrm_TransferSync(void) {
    return guard([&] { C().sync_xfer(); });
}
HB_API int helrm_GetPlaintextData(int pt, uint64_t *out, size_t words) {
    return guard([&] {
        Context &c = C();
        const Pt &p = c.pt(pt);
        size_t need = (size_t)(p.nq + (p.ext ? c.K : 0)) * c.N;
        if (!out || words < need) HB_THROW(HB_EINVAL, "GetPlaintextData: buffer too small");
        cuda_check(cudaMemcpyAsync(out, p.d, need * 8, cudaMemcpyDeviceToHost, c.stream), "d2h");
        c.sync();
    });
}
HB_API int helrm_NewPlaintextFromData(const uint64_t *data, int level, int ext, double scale, int *out) {
    return guard([&] {
        Context &c = C();
        OUT(out);
        if (level < 0 || level >= c.L || !data) HB_THROW(HB_EINVAL, "NewPlaintextFromData: bad level");
        Pt p;
        p.nq = level + 1;
        p.ext = ext != 0;
        p.scale = scale;
        p.slots = c.slots;
        size_t words = (size_t)(p.nq + (p.ext ? c.K : 0)) * c.N;
        p.d = c.alloc(words);
        cuda_check(cudaMemcpyAsync(p.d, data, words * 8, cudaMemcpyHostToDevice, c.stream), "h2d");
        c.sync();
        *out = c.put_pt(p);
    });
}
HB_API int helrm_GetKeyData(uint64_t galois, uint64_t *out, size_t words) {
    return guard([&] {
        Context &c = C();
        if (!out || words < c.key_words()) HB_THROW(HB_EINVAL, "GetKeyData: buffer too small");
        const u64 *k = nullptr;
        if (galois == 0) {
            if (!c.d_rlk) HB_THROW(HB_ENOENT, "no relinearisation key");
            k = c.d_rlk;
        } else {
            auto it = c.rot_keys.find(galois);
            if (it == c.rot_keys.end()) HB_THROW(HB_ENOENT, "no key for this Galois element");
            k = it->second;
        }
        cuda_check(cudaMemcpyAsync(out, k, c.key_words() * 8, cudaMemcpyDeviceToHost, c.stream), "d2h");
        c.sync();
    });
}
HB_API int helrm_GetSecretKeyData(uint64_t *out, size_t words) {
    return guard([&] {
        Context &c = C();
        c.require_sk();
        if (!out || words < (size_t)c.P * c.N) HB_THROW(HB_EINVAL, "GetSecretKeyData: buffer too small");
        cuda_check(cudaMemcpyAsync(out, c.d_sk, (size_t)c.P * c.N * 8, cudaMemcpyDeviceToHost, c.stream), "d2h");
        c.sync();
    });
}
HB_API int helrm_GetLinearTransformPlaintext(int lt, int k, uint64_t *out, size_t words) {
    return guard([&] {
        Context &c = C();
        LinTrans &t = c.lt(lt);
        auto it = t.pts.find(k);
        if (it == t.pts.end()) HB_THROW(HB_ENOENT, "no such diagonal");
        size_t need = (size_t)(it->second.nq + c.K) * c.N;
        if (!out || words < need) HB_THROW(HB_EINVAL, "buffer too small");
        cuda_check(cudaMemcpyAsync(out, it->second.d, need * 8, cudaMemcpyDeviceToHost, c.stream), "d2h");
        c.sync();
    });
}

HB_API int helrm_kernel_ntt(uint64_t *d, int nrows, int per, int nq, int inverse, void *stream) {
    return guard([&] {
        Context &c = C();
        if (!d || nrows <= 0 || per <= 0 || nq < 0 || nq > c.L || per - nq > c.K)
            HB_THROW(HB_EINVAL, "kernel_ntt: bad arguments");
        cudaStream_t s = stream ? (cudaStream_t)stream : c.stream;
        if (inverse)
            ntt_inverse((u64 *)d, nrows, rowmap(per, nq, c.L), c.ntt, s);
        else
            ntt_forward((u64 *)d, nrows, rowmap(per, nq, c.L), c.ntt, s);
    });
}
HB_API int helrm_kernel_automorphism(const uint64_t *in, uint64_t *out, int nrows, uint64_t galois, void *stream) {
    return guard([&] {
        Context &c = C();
        if (!in || !out || nrows <= 0 || (galois & 1) == 0) HB_THROW(HB_EINVAL, "kernel_automorphism: bad arguments");
        ew_automorphism((u64 *)out, (const u64 *)in, nrows, galois % (2ull * c.N), c.logN,
                        stream ? (cudaStream_t)stream : c.stream);
    });
}
HB_API int helrm_kernel_rescale(const uint64_t *in, uint64_t *out, int nq, int nbatch, void *stream) {
    return guard([&] {
        Context &c = C();
        if (!in || !out || nq < 2 || nq > c.L || nbatch <= 0) HB_THROW(HB_EINVAL, "kernel_rescale: bad arguments");
        cudaStream_t old = c.stream;
        if (stream) c.stream = (cudaStream_t)stream;
        try {
            c.rescale((u64 *)out, (const u64 *)in, 2, nq, nbatch, (size_t)2 * nq * c.N, (size_t)2 * (nq - 1) * c.N);
        } catch (...) {
            c.stream = old;
            throw;
        }
        c.stream = old;
    });
}

// ---- rescale without device allocation ---------------------------------------
// (the scratch array itself and its address lookup sit above class Context)
HB_API int helrm_kernel_rescale_noalloc(const uint64_t *in, uint64_t *out, int nq, int nbatch, void *stream) {
    return guard([&] {
        Context &c = C();
        if (!in || !out || nq < 2 || nq > c.L || nbatch <= 0)
            HB_THROW(HB_EINVAL, "kernel_rescale_noalloc: bad arguments");
        const size_t need = (size_t)nbatch * 2 * nq * c.N;
        if (need > (size_t)HELRM_RESCALE_SCRATCH_WORDS)
            HB_THROW(HB_EINVAL, "kernel_rescale_noalloc: needs " + std::to_string(need) +
                                    " scratch words (nbatch*2*nq*N), above the static limit of " +
                                    std::to_string((size_t)HELRM_RESCALE_SCRATCH_WORDS));
        u64 *scratch = c.d_rescale_scratch;
        cudaStream_t old = c.stream;
        if (stream) c.stream = (cudaStream_t)stream;
        try {
            c.rescale_scratch((u64 *)out, (const u64 *)in, 2, nq, nbatch, (size_t)2 * nq * c.N,
                              (size_t)2 * (nq - 1) * c.N, scratch);
        } catch (...) {
            c.stream = old;
            throw;
        }
        c.stream = old;
    });
}
HB_API int helrm_kernel_mac(const uint64_t *const *cts, const uint64_t *const *pts, int nterms, int nq, uint64_t *out,
                            void *stream) {
    return guard([&] {
        Context &c = C();
        if (!cts || !pts || !out || nterms <= 0 || nterms > HB_MAC_MAX || nq <= 0 || nq > c.L)
            HB_THROW(HB_EINVAL, "kernel_mac: bad arguments");
        MacArgs m{};
        for (int t = 0; t < nterms; t++) {
            m.ct[t] = (const u64 *)cts[t];
            m.pt[t] = (const u64 *)pts[t];
        }
        m.n = nterms;
        ew_mac((u64 *)out, m, 2, nq, c.logN, stream ? (cudaStream_t)stream : c.stream);
    });
}
HB_API int helrm_kernel_rotate_hoisted(const uint64_t *in, int nq, int nbatch, const int *ks, int nrot, uint64_t *out,
                                       void *stream) {
    return guard([&] {
        Context &c = C();
        if (!in || !out || !ks || nq <= 0 || nq > c.L || nbatch <= 0 || nrot <= 0)
            HB_THROW(HB_EINVAL, "kernel_rotate_hoisted: bad arguments");
        std::vector<u64> gs;
        std::vector<u64 *> outs;
        const size_t per = (size_t)nbatch * 2 * nq * c.N;
        for (int r = 0; r < nrot; r++) {
            u64 g = c.galois_of(ks[r]);
            if (g == 1) HB_THROW(HB_EINVAL, "kernel_rotate_hoisted: zero shift");
            if (!c.rot_keys.count(g)) HB_THROW(HB_ESTATE, "kernel_rotate_hoisted: missing rotation key");
            gs.push_back(g);
            outs.push_back((u64 *)out + r * per);
        }
        cudaStream_t old = c.stream;
        if (stream) c.stream = (cudaStream_t)stream;
        try {
            c.rotate_hoisted((const u64 *)in, nq, nbatch, gs, outs, (size_t)2 * nq * c.N);
        } catch (...) {
            c.stream = old;
            throw;
        }
        c.stream = old;
    });
}
HB_API int helrm_Synchronize(void) {
    return guard([&] { C().sync(); });
}

// ---- measurement ----------------------------------------------------------
static cudaEvent_t g_t0 = nullptr, g_t1 = nullptr;

HB_API int helrm_TimerStart(void) {
    return guard([&] {
        Context &c = C();
        if (!g_t0) {
            cuda_check(cudaEventCreate(&g_t0), "event");
            cuda_check(cudaEventCreate(&g_t1), "event");
        }
        cuda_check(cudaEventRecord(g_t0, c.stream), "event record");
    });
}
HB_API int helrm_TimerStop(double *ms) {
    return guard([&] {
        Context &c = C();
        OUT(ms);
        if (!g_t0) HB_THROW(HB_ESTATE, "TimerStop without TimerStart");
        if (c.up) {  // the region ends after the transfers issued in it, too
            c.wait_for(c.stream, c.up, c.ev_up);
            c.wait_for(c.stream, c.dn, c.ev_dn);
        }
        cuda_check(cudaEventRecord(g_t1, c.stream), "event record");
        cuda_check(cudaEventSynchronize(g_t1), "event sync");
        float f = 0.f;
        cuda_check(cudaEventElapsedTime(&f, g_t0, g_t1), "elapsed");
        *ms = f;
    });
}
HB_API int helrm_ProfileEnable(int on) {
    return guard([&] {
        C().sync();
        prof_enable(on != 0);
    });
}
HB_API int helrm_ProfileRead(double *ms, double *bytes, double *work, uint64_t *launches, int cap, int *nclasses) {
    return guard([&] {
        C().sync();
        ProfStats st;
        prof_collect(&st);
        if (nclasses) *nclasses = KC_COUNT;
        for (int i = 0; i < KC_COUNT && i < cap; i++) {
            if (ms) ms[i] = st.ms[i];
            if (bytes) bytes[i] = st.bytes[i];
            if (work) work[i] = st.work[i];
            if (launches) launches[i] = st.launches[i];
        }
    });
}
HB_API int helrm_KernelClassName(int cls, char *out, int cap) {
    return guard([&] {
        if (!out || cap <= 0) HB_THROW(HB_EINVAL, "KernelClassName: bad buffer");
        std::snprintf(out, (size_t)cap, "%s", kclass_name(cls));
    });
}
HB_API int helrm_ProfilerRange(int on) {
    return guard([&] {
        C().sync();
        cuda_check(on ? cudaProfilerStart() : cudaProfilerStop(), "profiler range");
    });
}
HB_API int helrm_GetLaunchCount(uint64_t *n) {
    return guard([&] {
        OUT(n);
        *n = launch_count();
    });
}
HB_API int helrm_GetAllocCount(uint64_t *n) {
    return guard([&] {
        OUT(n);
        *n = C().n_allocs;
    });
}
