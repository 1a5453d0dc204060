// hb_kernels.cu -- sm_100a kernels of the B200 CKKS backend.
//
// All residues are 64-bit words below q < 2^61, limb-major in HBM.  The
// kernels are integer CUDA-core code: modular arithmetic is not a dense
// MMA, so no tensor cores are involved.  Data that a kernel reads more
// than once per thread block (NTT twiddle tiles, the per-chunk baby-step
// descriptors) is staged in shared memory; everything else streams with
// 16-byte vector accesses.
#include <cooperative_groups.h>
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <vector>

#include "hb_kernels.cuh"

namespace hb {

__constant__ PrimeConst c_pc[HB_MAX_PRIMES];
}  // namespace hb

#include "hb_bsgs.cuh"
#include "hb_bsgs_tc.cuh"

namespace hb {

static void check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// host copy of the moduli in the constant table (launchers pick kernel
// specialisations by prime size)
static u64 g_host_q[HB_MAX_PRIMES];
static int g_host_nq = 0;

void upload_prime_consts(const PrimeConst *pc, int n) {
    cudaError_t e = cudaMemcpyToSymbol(c_pc, pc, sizeof(PrimeConst) * n);
    if (e != cudaSuccess) throw std::runtime_error(std::string("prime constants: ") + cudaGetErrorString(e));
    for (int i = 0; i < n; i++) g_host_q[i] = pc[i].q;
    g_host_nq = n;
}

// every prime p0 .. p0 + n - 1 of the table below 2^40 (below = true) or
// every one at or above it (below = false)
static bool primes_sized(int p0, int n, bool below) {
    if (p0 < 0 || p0 + n > g_host_nq) return false;
    for (int i = p0; i < p0 + n; i++)
        if ((g_host_q[i] < (1ull << 40)) != below) return false;
    return true;
}

// =====================================================================
// Launch accounting.  Every launcher counts the kernels it launches and,
// while profiling is on, brackets them with CUDA events on the stream it
// launches on, tagged with the launch's algorithmic bytes (each operand
// read or written once) and integer work (modular products, or NTT
// butterflies).  prof_collect() resolves the events.
// =====================================================================
static unsigned long long g_launches = 0;
static bool g_prof_on = false;
struct ProfRec {
    cudaEvent_t a, b;
    int cls;
    double bytes, work;
};
static std::vector<ProfRec> g_pending;
static std::vector<cudaEvent_t> g_event_pool;
static ProfStats g_stats;

static cudaEvent_t pool_event() {
    if (!g_event_pool.empty()) {
        cudaEvent_t e = g_event_pool.back();
        g_event_pool.pop_back();
        return e;
    }
    cudaEvent_t e;
    cudaEventCreate(&e);
    return e;
}

struct ProfScope {
    int cls;
    double bytes, work;
    cudaStream_t s;
    cudaEvent_t a = nullptr;
    ProfScope(int c, double by, double wk, cudaStream_t st, int nlaunch) : cls(c), bytes(by), work(wk), s(st) {
        g_launches += (unsigned long long)nlaunch;
        if (g_prof_on) {
            a = pool_event();
            cudaEventRecord(a, s);
        }
    }
    ~ProfScope() {
        if (a) {
            cudaEvent_t b = pool_event();
            cudaEventRecord(b, s);
            g_pending.push_back({a, b, cls, bytes, work});
        }
    }
};

static const char *kClassNames[KC_COUNT] = {
    "ntt_forward", "ntt_inverse", "modup_bconv", "moddown_bconv", "moddown_combine", "keymult",
    "bsgs_baby_mac", "rescale", "elementwise", "automorphism", "sampling", "bsgs_mac_mma"};

const char *kclass_name(int c) { return (c >= 0 && c < KC_COUNT) ? kClassNames[c] : ""; }
unsigned long long launch_count() { return g_launches; }

void prof_collect(ProfStats *out) {
    for (auto &r : g_pending) {
        cudaEventSynchronize(r.b);
        float ms = 0.f;
        cudaEventElapsedTime(&ms, r.a, r.b);
        g_stats.ms[r.cls] += ms;
        g_stats.bytes[r.cls] += r.bytes;
        g_stats.work[r.cls] += r.work;
        g_stats.launches[r.cls] += 1;
        g_event_pool.push_back(r.a);
        g_event_pool.push_back(r.b);
    }
    g_pending.clear();
    if (out) *out = g_stats;
}

void prof_enable(bool on) {
    prof_collect(nullptr);
    g_stats = ProfStats{};
    g_prof_on = on;
}

static inline unsigned grid1d(size_t work, int block) {
    size_t g = (work + block - 1) / block;
    return (unsigned)(g ? g : 1);
}

// =====================================================================
// NTT.  N = N1 * N2.  Forward (Cooley-Tukey, bit-reversed output): the
// first log2(N1) stages pair elements N2 apart and stay inside a column
// {k*N2 + c}; the last log2(N2) stages stay inside a contiguous block of
// N2.  Pass 1 runs the column stages on a tile of C columns, pass 2 the
// block stages on RB blocks; each pass stages its tile in shared memory.
// The inverse (Gentleman-Sande) runs the block stages first.
// =====================================================================
static inline int split_log1(int logN) { return logN / 2; }

// Radix-4 rounds: a thread owns the four elements {j, j+t/2, j+t, j+3t/2}
// of a group of 2t and applies two consecutive stages to them in registers
// (one shared-memory round trip per two stages).  Forward butterflies are
// Harvey's lazy form with values in [0, 4q); the inverse keeps [0, 2q); the
// store reduces fully.
__device__ __forceinline__ void ct_bfly(u64 &x, u64 &y, u64 w, u64 wp, u64 q) {
    const u64 two_q = 2 * q;
    if (x >= two_q) x -= two_q;
    const u64 t = mul_shoup_lazy(y, w, wp, q);
    y = x + two_q - t;
    x = x + t;
}
__device__ __forceinline__ void gs_bfly(u64 &x, u64 &y, u64 w, u64 wp, u64 q) {
    const u64 two_q = 2 * q;
    u64 s = x + y;
    if (s >= two_q) s -= two_q;
    const u64 d = x + two_q - y;
    x = s;
    y = mul_shoup_lazy(d, w, wp, q);
}
__device__ __forceinline__ u64 reduce4q(u64 x, u64 q) {
    if (x >= 2 * q) x -= 2 * q;
    if (x >= q) x -= q;
    return x;
}

// Stage s of an n-point transform on a shared-memory tile addressed by
// idx(k): forward stage with m groups pairs k and k + n/(2m); twiddle of
// group i is tw[wbase(m) + i].
template <bool INV>
__global__ void __launch_bounds__(256) k_ntt_cols(u64 *__restrict__ data, RowMap map, const u64 *__restrict__ tw,
                                                   const u64 *__restrict__ twp, int logN, int logN1, int logC,
                                                   int row0) {
    extern __shared__ u64 sm[];
    const int row = row0 + blockIdx.y;
    if (map.skip(row)) return;
    const int p = map.prime(row);
    const u64 q = c_pc[p].q;
    const int N = 1 << logN, N1 = 1 << logN1, N2 = N >> logN1, C = 1 << logC;
    const int c0 = blockIdx.x << logC;
    u64 *a = data + (size_t)row * N;
    const u64 *W = tw + (size_t)p * N, *Wp = twp + (size_t)p * N;
    for (int idx = threadIdx.x; idx < (N1 << logC); idx += blockDim.x) {
        int kk = idx >> logC, c = idx & (C - 1);
        sm[idx] = a[(size_t)kk * N2 + c0 + c];
    }
    __syncthreads();
#define SMC(kk) sm[((kk) << logC) + c]
    if (!INV) {
        int lt = logN1 - 1;  // log2 of the half distance t at the current stage
        int m = 1;
        for (; lt >= 1; lt -= 2, m <<= 2) {
            const int nq4 = (N1 >> 2) << logC;
            for (int u = threadIdx.x; u < nq4; u += blockDim.x) {
                const int c = u & (C - 1), j = u >> logC;
                const int t = 1 << lt, h = t >> 1;
                const int i = j >> (lt - 1), jj = j & (h - 1);
                const int k0 = (i << (lt + 1)) + jj;
                u64 x0 = SMC(k0), x1 = SMC(k0 + h), x2 = SMC(k0 + t), x3 = SMC(k0 + t + h);
                const u64 w1 = __ldg(W + m + i), w1p = __ldg(Wp + m + i);
                ct_bfly(x0, x2, w1, w1p, q);
                ct_bfly(x1, x3, w1, w1p, q);
                const u64 w2 = __ldg(W + 2 * m + 2 * i), w2p = __ldg(Wp + 2 * m + 2 * i);
                const u64 w3 = __ldg(W + 2 * m + 2 * i + 1), w3p = __ldg(Wp + 2 * m + 2 * i + 1);
                ct_bfly(x0, x1, w2, w2p, q);
                ct_bfly(x2, x3, w3, w3p, q);
                SMC(k0) = x0;
                SMC(k0 + h) = x1;
                SMC(k0 + t) = x2;
                SMC(k0 + t + h) = x3;
            }
            __syncthreads();
        }
        if (lt == 0) {  // odd number of stages: one radix-2 round
            const int nb2 = (N1 >> 1) << logC;
            for (int u = threadIdx.x; u < nb2; u += blockDim.x) {
                const int c = u & (C - 1), i = u >> logC;
                u64 x0 = SMC(2 * i), x1 = SMC(2 * i + 1);
                ct_bfly(x0, x1, __ldg(W + m + i), __ldg(Wp + m + i), q);
                SMC(2 * i) = x0;
                SMC(2 * i + 1) = x1;
            }
            __syncthreads();
        }
        for (int idx = threadIdx.x; idx < (N1 << logC); idx += blockDim.x) {
            int kk = idx >> logC, c = idx & (C - 1);
            a[(size_t)kk * N2 + c0 + c] = reduce4q(sm[idx], q);
        }
    } else {
        int lt = 0;
        int h = N1 >> 1;  // groups at the current stage
        if (logN1 & 1) {  // odd: one radix-2 round first (t = 1)
            const int nb2 = (N1 >> 1) << logC;
            for (int u = threadIdx.x; u < nb2; u += blockDim.x) {
                const int c = u & (C - 1), i = u >> logC;
                u64 x0 = SMC(2 * i), x1 = SMC(2 * i + 1);
                gs_bfly(x0, x1, __ldg(W + h + i), __ldg(Wp + h + i), q);
                SMC(2 * i) = x0;
                SMC(2 * i + 1) = x1;
            }
            __syncthreads();
            lt = 1;
            h >>= 1;
        }
        for (; lt < logN1; lt += 2, h >>= 2) {
            const int nq4 = (N1 >> 2) << logC;
            for (int u = threadIdx.x; u < nq4; u += blockDim.x) {
                const int c = u & (C - 1), j = u >> logC;
                const int t = 1 << lt;  // first stage half distance
                const int i2 = j >> lt, jj = j & (t - 1);  // group of the second stage (distance 2t)
                const int k0 = (i2 << (lt + 2)) + jj;
                u64 x0 = SMC(k0), x1 = SMC(k0 + t), x2 = SMC(k0 + 2 * t), x3 = SMC(k0 + 3 * t);
                const int i1 = 2 * i2;  // groups of the first stage: i1, i1+1
                gs_bfly(x0, x1, __ldg(W + h + i1), __ldg(Wp + h + i1), q);
                gs_bfly(x2, x3, __ldg(W + h + i1 + 1), __ldg(Wp + h + i1 + 1), q);
                const int hh = h >> 1;
                gs_bfly(x0, x2, __ldg(W + hh + i2), __ldg(Wp + hh + i2), q);
                gs_bfly(x1, x3, __ldg(W + hh + i2), __ldg(Wp + hh + i2), q);
                SMC(k0) = x0;
                SMC(k0 + t) = x1;
                SMC(k0 + 2 * t) = x2;
                SMC(k0 + 3 * t) = x3;
            }
            __syncthreads();
        }
        const u64 ni = c_pc[p].ninv, nip = c_pc[p].ninvp;
        for (int idx = threadIdx.x; idx < (N1 << logC); idx += blockDim.x) {
            int kk = idx >> logC, c = idx & (C - 1);
            a[(size_t)kk * N2 + c0 + c] = mul_shoup(sm[idx], ni, nip, q);
        }
    }
#undef SMC
}

template <bool INV>
__global__ void __launch_bounds__(256) k_ntt_rows(u64 *__restrict__ data, RowMap map, const u64 *__restrict__ tw,
                                                   const u64 *__restrict__ twp, int logN, int logN1, int logRB,
                                                   int row0) {
    extern __shared__ u64 sm[];
    const int row = row0 + blockIdx.y;
    if (map.skip(row)) return;
    const int p = map.prime(row);
    const u64 q = c_pc[p].q;
    const int N = 1 << logN, N1 = 1 << logN1, logN2 = logN - logN1, N2 = 1 << logN2;
    const int rb0 = blockIdx.x << logRB;
    const int tile = N2 << logRB;
    u64 *a = data + (size_t)row * N + (size_t)rb0 * N2;
    const u64 *W = tw + (size_t)p * N, *Wp = twp + (size_t)p * N;
    {
        const ulonglong2 *src = reinterpret_cast<const ulonglong2 *>(a);
        ulonglong2 *dst = reinterpret_cast<ulonglong2 *>(sm);
        for (int idx = threadIdx.x; idx < (tile >> 1); idx += blockDim.x) dst[idx] = src[idx];
    }
    __syncthreads();
    const int nq4 = (N2 >> 2) << logRB;
    if (!INV) {
        // forward stage with mp groups per block: twiddle of (block rb, group i) at mp*(N1 + rb) + i
        int lt = logN2 - 1, mp = 1;
        for (; lt >= 1; lt -= 2, mp <<= 2) {
            for (int u = threadIdx.x; u < nq4; u += blockDim.x) {
                const int blk = u >> (logN2 - 2), j = u & ((N2 >> 2) - 1);
                const int t = 1 << lt, h = t >> 1;
                const int i = j >> (lt - 1), jj = j & (h - 1);
                const int k0 = (blk << logN2) + (i << (lt + 1)) + jj;
                const int rb = rb0 + blk;
                u64 x0 = sm[k0], x1 = sm[k0 + h], x2 = sm[k0 + t], x3 = sm[k0 + t + h];
                const int w1i = mp * (N1 + rb) + i;
                ct_bfly(x0, x2, __ldg(W + w1i), __ldg(Wp + w1i), q);
                ct_bfly(x1, x3, __ldg(W + w1i), __ldg(Wp + w1i), q);
                const int w2i = 2 * mp * (N1 + rb) + 2 * i;
                ct_bfly(x0, x1, __ldg(W + w2i), __ldg(Wp + w2i), q);
                ct_bfly(x2, x3, __ldg(W + w2i + 1), __ldg(Wp + w2i + 1), q);
                sm[k0] = x0;
                sm[k0 + h] = x1;
                sm[k0 + t] = x2;
                sm[k0 + t + h] = x3;
            }
            __syncthreads();
        }
        if (lt == 0) {
            const int nb2 = (N2 >> 1) << logRB;
            for (int u = threadIdx.x; u < nb2; u += blockDim.x) {
                const int blk = u >> (logN2 - 1), i = u & ((N2 >> 1) - 1);
                const int k0 = (blk << logN2) + 2 * i;
                const int wi = mp * (N1 + rb0 + blk) + i;
                u64 x0 = sm[k0], x1 = sm[k0 + 1];
                ct_bfly(x0, x1, __ldg(W + wi), __ldg(Wp + wi), q);
                sm[k0] = x0;
                sm[k0 + 1] = x1;
            }
            __syncthreads();
        }
    } else {
        int lt = 0, hp = N2 >> 1;
        if (logN2 & 1) {
            const int nb2 = (N2 >> 1) << logRB;
            for (int u = threadIdx.x; u < nb2; u += blockDim.x) {
                const int blk = u >> (logN2 - 1), i = u & ((N2 >> 1) - 1);
                const int k0 = (blk << logN2) + 2 * i;
                const int wi = hp * (N1 + rb0 + blk) + i;
                u64 x0 = sm[k0], x1 = sm[k0 + 1];
                gs_bfly(x0, x1, __ldg(W + wi), __ldg(Wp + wi), q);
                sm[k0] = x0;
                sm[k0 + 1] = x1;
            }
            __syncthreads();
            lt = 1;
            hp >>= 1;
        }
        for (; lt < logN2; lt += 2, hp >>= 2) {
            for (int u = threadIdx.x; u < nq4; u += blockDim.x) {
                const int blk = u >> (logN2 - 2), j = u & ((N2 >> 2) - 1);
                const int t = 1 << lt;
                const int i2 = j >> lt, jj = j & (t - 1);
                const int k0 = (blk << logN2) + (i2 << (lt + 2)) + jj;
                const int rb = rb0 + blk;
                u64 x0 = sm[k0], x1 = sm[k0 + t], x2 = sm[k0 + 2 * t], x3 = sm[k0 + 3 * t];
                const int i1 = 2 * i2;
                const int wa = hp * (N1 + rb) + i1;
                gs_bfly(x0, x1, __ldg(W + wa), __ldg(Wp + wa), q);
                gs_bfly(x2, x3, __ldg(W + wa + 1), __ldg(Wp + wa + 1), q);
                const int wb = (hp >> 1) * (N1 + rb) + i2;
                gs_bfly(x0, x2, __ldg(W + wb), __ldg(Wp + wb), q);
                gs_bfly(x1, x3, __ldg(W + wb), __ldg(Wp + wb), q);
                sm[k0] = x0;
                sm[k0 + t] = x1;
                sm[k0 + 2 * t] = x2;
                sm[k0 + 3 * t] = x3;
            }
            __syncthreads();
        }
        // the column pass reduces fully; values here stay in [0, 2q)
    }
    {
        const ulonglong2 *src = reinterpret_cast<const ulonglong2 *>(sm);
        ulonglong2 *dst = reinterpret_cast<ulonglong2 *>(a);
        for (int idx = threadIdx.x; idx < (tile >> 1); idx += blockDim.x) {
            ulonglong2 v = src[idx];
            if (!INV) {  // forward output fully reduced
                v.x = reduce4q(v.x, q);
                v.y = reduce4q(v.y, q);
            }
            dst[idx] = v;
        }
    }
}

// ---------------------------------------------------------------------
// N = 2^16 = 256 x 256: radix-16 passes.  A thread block owns 16
// sub-transforms of 256 points (16 columns in the column pass, 16
// contiguous blocks in the block pass) and 16 threads per sub-transform;
// each thread holds 16 elements in registers and runs 4 stages on them,
// the sub-transform is transposed through shared memory, and the thread
// runs the remaining 4 stages.  Twiddle of a stage with g groups per
// sub-transform, sub-transform sb of S: tw[g * (S + sb) + i].
//   layout A: the thread's elements are e = c + 16k (k = 0..15)
//   layout B: e = 16c + k
// ---------------------------------------------------------------------
// forward, layout A, groups 1, 2, 4, 8 (distances 128..16)
__device__ __forceinline__ void fwd_a(u64 (&x)[16], const u64 *W, const u64 *Wp, int base, u64 q) {
#pragma unroll
    for (int s = 0; s < 4; s++) {
        const int d = 8 >> s, g = 1 << s;
#pragma unroll
        for (int k = 0; k < 16; k++) {
            if (k & d) continue;
            const int i = k >> (4 - s);
            const int wi = g * base + i;
            ct_bfly(x[k], x[k + d], __ldg(W + wi), __ldg(Wp + wi), q);
        }
    }
}
// forward, layout B, groups 16, 32, 64, 128 (distances 8..1)
__device__ __forceinline__ void fwd_b(u64 (&x)[16], const u64 *W, const u64 *Wp, int base, int c, u64 q) {
#pragma unroll
    for (int s = 0; s < 4; s++) {
        const int d = 8 >> s, g = 16 << s;
#pragma unroll
        for (int k = 0; k < 16; k++) {
            if (k & d) continue;
            const int i = (c << s) + (k >> (4 - s));
            const int wi = g * base + i;
            ct_bfly(x[k], x[k + d], __ldg(W + wi), __ldg(Wp + wi), q);
        }
    }
}
// inverse, layout B, groups 128, 64, 32, 16 (distances 1..8)
__device__ __forceinline__ void inv_b(u64 (&x)[16], const u64 *W, const u64 *Wp, int base, int c, u64 q) {
#pragma unroll
    for (int s = 3; s >= 0; s--) {
        const int d = 8 >> s, g = 16 << s;
#pragma unroll
        for (int k = 0; k < 16; k++) {
            if (k & d) continue;
            const int i = (c << s) + (k >> (4 - s));
            const int wi = g * base + i;
            gs_bfly(x[k], x[k + d], __ldg(W + wi), __ldg(Wp + wi), q);
        }
    }
}
// inverse, layout A, groups 8, 4, 2, 1 (distances 16..128)
__device__ __forceinline__ void inv_a(u64 (&x)[16], const u64 *W, const u64 *Wp, int base, u64 q) {
#pragma unroll
    for (int s = 3; s >= 0; s--) {
        const int d = 8 >> s, g = 1 << s;
#pragma unroll
        for (int k = 0; k < 16; k++) {
            if (k & d) continue;
            const int i = k >> (4 - s);
            const int wi = g * base + i;
            gs_bfly(x[k], x[k + d], __ldg(W + wi), __ldg(Wp + wi), q);
        }
    }
}

// Forward butterflies in double precision (primes below 2^40).  Values are
// exact integers held as doubles, centred (possibly negative).  With
// Q = round(y fl(w/q)) (magic-number rounding), ph + pl = Q q exactly
// (TwoProduct: ph = fl(Q q), pl = fma(Q, q, -ph)), and fma(y, w, -ph) is the
// exact integer y w - ph (below 2^41 in magnitude), so
// t = y w - Q q = fma(y, w, -ph) - pl exactly, |t| <= 0.502 q for |y| < 2^44.
// x' = x + t, y' = x - t: magnitudes grow by 0.502 q per stage, below 9.1 q
// after 16 stages.  Eight FP64 instructions, no integer multiply: the FP64
// pipe is as fast as the integer-multiply pipe and otherwise idle.
__device__ __forceinline__ void ct_bfly_d(double &x, double &y, const double2 tw, double q) {
    const double magic = 6755399441055744.0;  // 1.5 * 2^52
    const double Qd = __dsub_rn(__fma_rn(y, tw.y, magic), magic);
    const double ph = __dmul_rn(Qd, q);
    const double pl = __fma_rn(Qd, q, -ph);
    const double t = __dsub_rn(__fma_rn(y, tw.x, -ph), pl);
    const double xn = __dadd_rn(x, t);
    y = __dsub_rn(x, t);
    x = xn;
}
template <bool G>
__device__ __forceinline__ double2 twld_d(const double2 *t, int i) {
    if (G) return __ldg(t + i);
    return t[i];
}
template <bool G>
__device__ __forceinline__ void fwd_a_d(double (&x)[16], const double2 *T, int base, double q) {
#pragma unroll
    for (int s = 0; s < 4; s++) {
        const int d = 8 >> s, g = 1 << s;
#pragma unroll
        for (int k = 0; k < 16; k++) {
            if (k & d) continue;
            ct_bfly_d(x[k], x[k + d], twld_d<G>(T, g * base + (k >> (4 - s))), q);
        }
    }
}
template <bool G>
__device__ __forceinline__ void fwd_b_d(double (&x)[16], const double2 *T, int base, int c, double q) {
#pragma unroll
    for (int s = 0; s < 4; s++) {
        const int d = 8 >> s, g = 16 << s;
#pragma unroll
        for (int k = 0; k < 16; k++) {
            if (k & d) continue;
            ct_bfly_d(x[k], x[k + d], twld_d<G>(T, g * base + (c << s) + (k >> (4 - s))), q);
        }
    }
}
// Inverse (Gentleman-Sande) butterflies in double precision: x' = x + y,
// y' = (x - y) w mod q (centred, as in ct_bfly_d).  Sums grow: from values
// below B a 4-stage group ends below 16 B, so every group ends by re-centring
// its 16 values to |v| <= 0.5 q; the first group starts from [0, q) and stays
// below 16 q < 2^44, the bound of the exact product.
__device__ __forceinline__ void gs_bfly_d(double &x, double &y, const double2 tw, double q) {
    const double sm = __dadd_rn(x, y);
    const double df = __dsub_rn(x, y);
    x = sm;
    y = mulmod_d(df, tw, q);
}
template <bool G>
__device__ __forceinline__ void inv_b_d(double (&x)[16], const double2 *T, int base, int c, double q, double qinv) {
#pragma unroll
    for (int s = 3; s >= 0; s--) {
        const int d = 8 >> s, g = 16 << s;
#pragma unroll
        for (int k = 0; k < 16; k++) {
            if (k & d) continue;
            gs_bfly_d(x[k], x[k + d], twld_d<G>(T, g * base + (c << s) + (k >> (4 - s))), q);
        }
    }
#pragma unroll
    for (int k = 0; k < 16; k++) x[k] = center_d(x[k], q, qinv);
}
// Block-pass twiddles as single doubles w; the pair {w, fl(w fl(1/q))} is
// formed in registers (the quotient estimate within 2^-12 of y w / q for
// |y| < 2^40, so a butterfly's |t| stays at most 0.5002 q).  NP values per
// thread: 1, 2 (one 128-bit load) or 4 (one 256-bit load) contiguous; 8 as
// two 256-bit loads STRIDE values apart.
template <int NP, int STRIDE>
__device__ __forceinline__ void ld_tw1(double2 (&tw)[8], const double *src, double qinv) {
    double w[8];
    if (NP == 1) {
        w[0] = __ldg(src);
    } else if (NP == 2) {
        const double2 v = __ldg(reinterpret_cast<const double2 *>(src));
        w[0] = v.x, w[1] = v.y;
    } else {
#pragma unroll
        for (int v = 0; v < NP / 4; v++)
            asm("ld.global.nc.v4.f64 {%0, %1, %2, %3}, [%4];"
                : "=d"(w[4 * v]), "=d"(w[4 * v + 1]), "=d"(w[4 * v + 2]), "=d"(w[4 * v + 3])
                : "l"(src + STRIDE * v));
    }
#pragma unroll
    for (int i = 0; i < NP; i++) tw[i] = make_double2(w[i], __dmul_rn(w[i], qinv));
}
__device__ __forceinline__ void fwd_a_ds(double (&x)[16], const double *T, int base, double q, double qinv) {
#pragma unroll
    for (int s = 0; s < 4; s++) {
        const int d = 8 >> s;
        double2 tw[8];
        if (s == 0) ld_tw1<1, 0>(tw, T + base, qinv);
        if (s == 1) ld_tw1<2, 0>(tw, T + 2 * base, qinv);
        if (s == 2) ld_tw1<4, 0>(tw, T + 4 * base, qinv);
        if (s == 3) ld_tw1<8, 4>(tw, T + 8 * base, qinv);
#pragma unroll
        for (int k = 0; k < 16; k++) {
            if (k & d) continue;
            ct_bfly_d(x[k], x[k + d], tw[k >> (4 - s)], q);
        }
    }
}
__device__ __forceinline__ void fwd_b_ds(double (&x)[16], const double *T, int base, int c, double q, double qinv) {
#pragma unroll
    for (int s = 0; s < 4; s++) {
        const int d = 8 >> s, g = 16 << s;
        double2 tw[8];
        const double *seg = T + g * base;
        if (s == 0) ld_tw1<1, 0>(tw, seg + c, qinv);
        if (s == 1) ld_tw1<2, 0>(tw, seg + 2 * c, qinv);
        if (s == 2) ld_tw1<4, 0>(tw, seg + 4 * c, qinv);
        if (s == 3) ld_tw1<8, 64>(tw, seg + 4 * c, qinv);
#pragma unroll
        for (int k = 0; k < 16; k++) {
            if (k & d) continue;
            ct_bfly_d(x[k], x[k + d], tw[k >> (4 - s)], q);
        }
    }
}
__device__ __forceinline__ void inv_b_ds(double (&x)[16], const double *T, int base, int c, double q, double qinv) {
#pragma unroll
    for (int s = 3; s >= 0; s--) {
        const int d = 8 >> s, g = 16 << s;
        double2 tw[8];
        const double *seg = T + g * base;
        if (s == 0) ld_tw1<1, 0>(tw, seg + c, qinv);
        if (s == 1) ld_tw1<2, 0>(tw, seg + 2 * c, qinv);
        if (s == 2) ld_tw1<4, 0>(tw, seg + 4 * c, qinv);
        if (s == 3) ld_tw1<8, 64>(tw, seg + 4 * c, qinv);
#pragma unroll
        for (int k = 0; k < 16; k++) {
            if (k & d) continue;
            gs_bfly_d(x[k], x[k + d], tw[k >> (4 - s)], q);
        }
    }
#pragma unroll
    for (int k = 0; k < 16; k++) x[k] = center_d(x[k], q, qinv);
}
__device__ __forceinline__ void inv_a_ds(double (&x)[16], const double *T, int base, double q, double qinv) {
#pragma unroll
    for (int s = 3; s >= 0; s--) {
        const int d = 8 >> s;
        double2 tw[8];
        if (s == 0) ld_tw1<1, 0>(tw, T + base, qinv);
        if (s == 1) ld_tw1<2, 0>(tw, T + 2 * base, qinv);
        if (s == 2) ld_tw1<4, 0>(tw, T + 4 * base, qinv);
        if (s == 3) ld_tw1<8, 4>(tw, T + 8 * base, qinv);
#pragma unroll
        for (int k = 0; k < 16; k++) {
            if (k & d) continue;
            gs_bfly_d(x[k], x[k + d], tw[k >> (4 - s)], q);
        }
    }
#pragma unroll
    for (int k = 0; k < 16; k++) x[k] = center_d(x[k], q, qinv);
}
template <bool G, bool CENTER>
__device__ __forceinline__ void inv_a_d(double (&x)[16], const double2 *T, int base, double q, double qinv) {
#pragma unroll
    for (int s = 3; s >= 0; s--) {
        const int d = 8 >> s, g = 1 << s;
#pragma unroll
        for (int k = 0; k < 16; k++) {
            if (k & d) continue;
            gs_bfly_d(x[k], x[k + d], twld_d<G>(T, g * base + (k >> (4 - s))), q);
        }
    }
    if (CENTER) {
#pragma unroll
        for (int k = 0; k < 16; k++) x[k] = center_d(x[k], q, qinv);
    }
}

// resident blocks per SM of the two 2^16 NTT passes
#ifndef HB_NTT_COLS_BLOCKS
#define HB_NTT_COLS_BLOCKS 4
#endif
#ifndef HB_NTT_ROWS_BLOCKS
#define HB_NTT_ROWS_BLOCKS 3
#endif
// Column pass: the 16 columns c0..c0+15, element (r, col) at r*256 + c0 + col.
// Primes below 2^40 take twiddle pairs {w, fl(w/q)} (the first 256
// entries, the same for every block, staged in shared memory); the others
// Shoup pairs from global memory.
template <bool INV>
__global__ void __launch_bounds__(256, HB_NTT_COLS_BLOCKS) k_ntt256_cols(u64 *__restrict__ data, RowMap map, const u64 *__restrict__ tw,
                                                      const u64 *__restrict__ twp,
                                                      const ulonglong2 *__restrict__ twx, int row0) {
    __shared__ u64 sm[256 * 17];
    __shared__ ulonglong2 stw[256];
    const int row = row0 + blockIdx.y;
    if (map.skip(row)) return;
    const int p = map.prime(row);
    const u64 q = c_pc[p].q;
    const bool fast = q < (1ull << 40);
    const int col = threadIdx.x & 15, c = threadIdx.x >> 4;
    const int c0 = blockIdx.x << 4;
    u64 *a = data + ((size_t)row << 16) + c0 + col;
    const u64 *W = tw + ((size_t)p << 16), *Wp = twp + ((size_t)p << 16);
    if (fast) stw[threadIdx.x] = __ldg(twx + ((size_t)p << 16) + threadIdx.x);
    u64 x[16];
    if (!INV && fast) {
        // double-precision butterflies; the block pass receives the centred
        // values as doubles (|v| < 5 q) and reduces at its end
        const double qd = (double)q;
        const double2 *stwd = reinterpret_cast<const double2 *>(stw);
        double xd[16];
#pragma unroll
        for (int k = 0; k < 16; k++) xd[k] = u64_to_d(a[(size_t)(c + 16 * k) << 8]);
        __syncthreads();
        fwd_a_d<false>(xd, stwd, 1, qd);
#pragma unroll
        for (int k = 0; k < 16; k++) sm[(c + 16 * k) * 17 + col] = (u64)__double_as_longlong(xd[k]);
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) xd[k] = __longlong_as_double((long long)sm[(16 * c + k) * 17 + col]);
        fwd_b_d<false>(xd, stwd, 1, c, qd);
#pragma unroll
        for (int k = 0; k < 16; k++) a[(size_t)(16 * c + k) << 8] = (u64)__double_as_longlong(xd[k]);
    } else if (!INV) {
        // primes of 40 bits and more: Harvey's lazy butterflies in [0, 4q)
#pragma unroll
        for (int k = 0; k < 16; k++) x[k] = a[(size_t)(c + 16 * k) << 8];
        fwd_a(x, W, Wp, 1, q);
#pragma unroll
        for (int k = 0; k < 16; k++) sm[(c + 16 * k) * 17 + col] = x[k];
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) x[k] = sm[(16 * c + k) * 17 + col];
        fwd_b(x, W, Wp, 1, c, q);
#pragma unroll
        for (int k = 0; k < 16; k++) a[(size_t)(16 * c + k) << 8] = reduce4q(x[k], q);
    } else if (fast) {
        // second pass of the double-precision inverse: doubles from the block
        // pass (|v| <= 0.5 q), the last 8 stages, then the factor N^-1
        const double qd = (double)q, qinv = c_pc[p].qinv;
        const double2 *stwd = reinterpret_cast<const double2 *>(stw);
        double xd[16];
#pragma unroll
        for (int k = 0; k < 16; k++) xd[k] = __longlong_as_double((long long)a[(size_t)(16 * c + k) << 8]);
        __syncthreads();
        inv_b_d<false>(xd, stwd, 1, c, qd, qinv);
#pragma unroll
        for (int k = 0; k < 16; k++) sm[(16 * c + k) * 17 + col] = (u64)__double_as_longlong(xd[k]);
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) xd[k] = __longlong_as_double((long long)sm[(c + 16 * k) * 17 + col]);
        inv_a_d<false, false>(xd, stwd, 1, qd, qinv);
        const double nid = (double)c_pc[p].ninv;
        const double2 ni = make_double2(nid, __ddiv_rn(nid, qd));
#pragma unroll
        for (int k = 0; k < 16; k++) {
            double r = mulmod_d(xd[k], ni, qd);  // |r| <= 0.502 q
            if (r < 0.0) r = __dadd_rn(r, qd);
            a[(size_t)(c + 16 * k) << 8] =
                (u64)__double_as_longlong(__dadd_rn(r, 4503599627370496.0)) & 0x000FFFFFFFFFFFFFull;
        }
    } else {
        // primes of 40 bits and more: Gentleman-Sande values in [0, 2q)
#pragma unroll
        for (int k = 0; k < 16; k++) x[k] = a[(size_t)(16 * c + k) << 8];
        inv_b(x, W, Wp, 1, c, q);
#pragma unroll
        for (int k = 0; k < 16; k++) sm[(16 * c + k) * 17 + col] = x[k];
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) x[k] = sm[(c + 16 * k) * 17 + col];
        inv_a(x, W, Wp, 1, q);
        const u64 ni = c_pc[p].ninv, nip = c_pc[p].ninvp;
#pragma unroll
        for (int k = 0; k < 16; k++) a[(size_t)(c + 16 * k) << 8] = mul_shoup(x[k], ni, nip, q);
    }
}

// Block pass: blocks rb0..rb0+15 of 256 contiguous elements.
template <bool INV>
__global__ void __launch_bounds__(256, HB_NTT_ROWS_BLOCKS) k_ntt256_rows(u64 *__restrict__ data, RowMap map, const u64 *__restrict__ tw,
                                                      const u64 *__restrict__ twp,
                                                      const ulonglong2 *__restrict__ twx,
                                                      const double *__restrict__ tws, int row0,
                                                      const u64 *__restrict__ src = nullptr, size_t src_stride = 0,
                                                      int src_per = 1) {
    __shared__ u64 sm[16 * 272];
    const int row = row0 + blockIdx.y;
    if (map.skip(row)) return;
    const int p = map.prime(row);
    const u64 q = c_pc[p].q;
    const bool fast = q < (1ull << 40);
    const int c = threadIdx.x & 15, blk = threadIdx.x >> 4;
    const int rb = (blockIdx.x << 4) + blk;
    u64 *a = data + ((size_t)row << 16) + ((size_t)rb << 8);
    const u64 *W = tw + ((size_t)p << 16), *Wp = twp + ((size_t)p << 16);
    u64 *sb = sm + blk * 272;  // 256 elements of this block, 17-word rows of 16 (padding)
    u64 x[16];
    if (!INV && fast) {
        // doubles from the column pass; reduced and converted at the end
        const double qd = (double)q, qinv = c_pc[p].qinv;
        double xd[16];
#pragma unroll
        for (int k = 0; k < 16; k++) xd[k] = __longlong_as_double((long long)a[c + 16 * k]);
        const double *Ts = tws + ((size_t)p << 16);
        fwd_a_ds(xd, Ts, 256 + rb, qd, qinv);
#pragma unroll
        for (int k = 0; k < 16; k++) sb[k * 17 + c] = (u64)__double_as_longlong(xd[k]);
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) xd[k] = __longlong_as_double((long long)sb[c * 17 + k]);
        fwd_b_ds(xd, Ts, 256 + rb, c, qd, qinv);
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) sb[c * 17 + k] = d_mod_to_u64(xd[k], qd, qinv);
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) a[c + 16 * k] = sb[k * 17 + c];
    } else if (!INV) {
        // primes of 40 bits and more: Harvey's lazy butterflies in [0, 4q)
#pragma unroll
        for (int k = 0; k < 16; k++) x[k] = a[c + 16 * k];
        fwd_a(x, W, Wp, 256 + rb, q);
#pragma unroll
        for (int k = 0; k < 16; k++) sb[k * 17 + c] = x[k];  // element c + 16k at (k, c)
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) x[k] = sb[c * 17 + k];  // element 16c + k
        fwd_b(x, W, Wp, 256 + rb, c, q);
#pragma unroll
        for (int k = 0; k < 16; k++) x[k] = reduce4q(x[k], q);
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) sb[c * 17 + k] = x[k];
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) a[c + 16 * k] = sb[k * 17 + c];
    } else {
        // out of place: the first (block) pass of the inverse reads row `row`
        // of the source, item row / src_per at src_stride, limb row % src_per
        const u64 *ain = src ? src + (size_t)(row / src_per) * src_stride + ((size_t)(row % src_per) << 16) +
                                   ((size_t)rb << 8)
                             : a;
#pragma unroll
        for (int k = 0; k < 16; k++) sb[k * 17 + c] = ain[c + 16 * k];
        __syncthreads();
        if (fast) {
            // first pass of the double-precision inverse; the column pass
            // receives centred doubles (|v| <= 0.5 q)
            const double qd = (double)q, qinv = c_pc[p].qinv;
            double xd[16];
#pragma unroll
            for (int k = 0; k < 16; k++) xd[k] = u64_to_d(sb[c * 17 + k]);
            const double *Ts = tws + ((size_t)p << 16);
            inv_b_ds(xd, Ts, 256 + rb, c, qd, qinv);
            __syncthreads();
#pragma unroll
            for (int k = 0; k < 16; k++) sb[c * 17 + k] = (u64)__double_as_longlong(xd[k]);
            __syncthreads();
#pragma unroll
            for (int k = 0; k < 16; k++) xd[k] = __longlong_as_double((long long)sb[k * 17 + c]);
            inv_a_ds(xd, Ts, 256 + rb, qd, qinv);
#pragma unroll
            for (int k = 0; k < 16; k++) a[c + 16 * k] = (u64)__double_as_longlong(xd[k]);
        } else {
#pragma unroll
            for (int k = 0; k < 16; k++) x[k] = sb[c * 17 + k];
            inv_b(x, W, Wp, 256 + rb, c, q);
            __syncthreads();
#pragma unroll
            for (int k = 0; k < 16; k++) sb[c * 17 + k] = x[k];
            __syncthreads();
#pragma unroll
            for (int k = 0; k < 16; k++) x[k] = sb[k * 17 + c];
            inv_a(x, W, Wp, 256 + rb, q);
#pragma unroll
            for (int k = 0; k < 16; k++) a[c + 16 * k] = x[k];  // [0, 2q): the column pass reduces
        }
    }
}

// One-pass 2^16 NTT: a cluster of 8 CTAs holds one limb in shared memory.
// CTA k runs the column pass on columns [32k, 32k+32) (two groups of 16,
// exactly the two-pass kernel's arithmetic), leaves the column-transformed
// values in its shared memory, and after a cluster barrier the row pass on
// rows [32k, 32k+32) reads its 256 columns from the 8 CTAs' shared memory
// (distributed shared memory, all within this GPU).  The inverse runs the
// row pass first.  The limb crosses HBM once each way instead of twice, and
// every butterfly is the two-pass kernels' own, so the results are
// identical.  Shared memory: one region reused by the column transposes,
// the exchange tile and the row transposes (barriers between the uses).
constexpr int kNttCl = 8;                     // CTAs per limb
constexpr int kNttClWords = 2 * 256 * 17;     // 8704 words: max of the three uses
constexpr int kNttXS = 33;                    // forward exchange tile row stride ([256][32])
constexpr int kNttXSi = 257;                  // inverse exchange tile row stride ([32][256])

template <bool INV>
__global__ void __cluster_dims__(kNttCl, 1, 1) __launch_bounds__(512, 2)
    k_ntt_cl(u64 *__restrict__ data, RowMap map, const u64 *__restrict__ tw, const u64 *__restrict__ twp,
             const ulonglong2 *__restrict__ twx, const double *__restrict__ tws, int row0,
             const u64 *__restrict__ src, size_t src_stride, int src_per) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ u64 shm[];
    __shared__ ulonglong2 stw[256];
    const int row = row0 + blockIdx.y;
    if (map.skip(row)) return;  // uniform over the cluster (same row)
    const int k = (int)cluster.block_rank();
    const int t = threadIdx.x;
    const int p = map.prime(row);
    const u64 q = c_pc[p].q;
    const bool fast = q < (1ull << 40);
    const double qd = (double)q, qinv = c_pc[p].qinv;
    const u64 *W = tw + ((size_t)p << 16), *Wp = twp + ((size_t)p << 16);
    const double *Ts = tws + ((size_t)p << 16);
    const double2 *stwd = reinterpret_cast<const double2 *>(stw);
    u64 *limb = data + ((size_t)row << 16);
    if (fast && t < 256) stw[t] = __ldg(twx + ((size_t)p << 16) + t);
    // column-pass roles: group g of 16 columns, column col, row phase c
    const int g = t >> 8, tt = t & 255, col = tt & 15, c = tt >> 4;
    const int gc = 32 * k + 16 * g + col;
    u64 *T = shm + g * 256 * 17;
    // row-pass roles: local row blk, phase cr
    const int blk = t >> 4, cr = t & 15;
    const int rb = 32 * k + blk;
    u64 *sb = shm + blk * 272;
    double xd[16];
    u64 x[16];
    if (!INV) {
        // ---- column pass (rows c + 16j of column gc)
        if (fast) {
#pragma unroll
            for (int j = 0; j < 16; j++) xd[j] = u64_to_d(limb[((size_t)(c + 16 * j) << 8) + gc]);
            __syncthreads();  // stw
            fwd_a_d<false>(xd, stwd, 1, qd);
#pragma unroll
            for (int j = 0; j < 16; j++) T[(c + 16 * j) * 17 + col] = (u64)__double_as_longlong(xd[j]);
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) xd[j] = __longlong_as_double((long long)T[(16 * c + j) * 17 + col]);
            fwd_b_d<false>(xd, stwd, 1, c, qd);
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) shm[(16 * c + j) * kNttXS + 16 * g + col] = (u64)__double_as_longlong(xd[j]);
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) x[j] = limb[((size_t)(c + 16 * j) << 8) + gc];
            fwd_a(x, W, Wp, 1, q);
#pragma unroll
            for (int j = 0; j < 16; j++) T[(c + 16 * j) * 17 + col] = x[j];
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) x[j] = T[(16 * c + j) * 17 + col];
            fwd_b(x, W, Wp, 1, c, q);
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) shm[(16 * c + j) * kNttXS + 16 * g + col] = reduce4q(x[j], q);
        }
        cluster.sync();
        // ---- row pass: row rb, columns cr + 16j from CTA j / 2
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const u64 *px = cluster.map_shared_rank(shm, j >> 1);
            x[j] = px[rb * kNttXS + cr + 16 * (j & 1)];
        }
        cluster.sync();  // every remote read done: the region is free again
        if (fast) {
#pragma unroll
            for (int j = 0; j < 16; j++) xd[j] = __longlong_as_double((long long)x[j]);
            fwd_a_ds(xd, Ts, 256 + rb, qd, qinv);
#pragma unroll
            for (int j = 0; j < 16; j++) sb[j * 17 + cr] = (u64)__double_as_longlong(xd[j]);
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) xd[j] = __longlong_as_double((long long)sb[cr * 17 + j]);
            fwd_b_ds(xd, Ts, 256 + rb, cr, qd, qinv);
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) sb[cr * 17 + j] = d_mod_to_u64(xd[j], qd, qinv);
        } else {
            fwd_a(x, W, Wp, 256 + rb, q);
#pragma unroll
            for (int j = 0; j < 16; j++) sb[j * 17 + cr] = x[j];
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) x[j] = sb[cr * 17 + j];
            fwd_b(x, W, Wp, 256 + rb, cr, q);
#pragma unroll
            for (int j = 0; j < 16; j++) x[j] = reduce4q(x[j], q);
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) sb[cr * 17 + j] = x[j];
        }
        __syncthreads();
        u64 *a = limb + ((size_t)rb << 8);
#pragma unroll
        for (int j = 0; j < 16; j++) a[cr + 16 * j] = sb[j * 17 + cr];
    } else {
        // ---- row pass first (row rb, from src when given)
        const u64 *ain = src ? src + (size_t)(row / src_per) * src_stride + ((size_t)(row % src_per) << 16) +
                                   ((size_t)rb << 8)
                             : limb + ((size_t)rb << 8);
#pragma unroll
        for (int j = 0; j < 16; j++) sb[j * 17 + cr] = ain[cr + 16 * j];
        __syncthreads();
        u64 *X = shm + blk * kNttXSi;  // local row blk of the exchange tile [32][256]
        if (fast) {
#pragma unroll
            for (int j = 0; j < 16; j++) xd[j] = u64_to_d(sb[cr * 17 + j]);
            inv_b_ds(xd, Ts, 256 + rb, cr, qd, qinv);
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) sb[cr * 17 + j] = (u64)__double_as_longlong(xd[j]);
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) xd[j] = __longlong_as_double((long long)sb[j * 17 + cr]);
            inv_a_ds(xd, Ts, 256 + rb, qd, qinv);
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) X[cr + 16 * j] = (u64)__double_as_longlong(xd[j]);
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) x[j] = sb[cr * 17 + j];
            inv_b(x, W, Wp, 256 + rb, cr, q);
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) sb[cr * 17 + j] = x[j];
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) x[j] = sb[j * 17 + cr];
            inv_a(x, W, Wp, 256 + rb, q);
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) X[cr + 16 * j] = x[j];
        }
        cluster.sync();
        // ---- column pass: column gc, rows 16c + j, all in CTA c / 2
        {
            const u64 *px = cluster.map_shared_rank(shm, c >> 1);
#pragma unroll
            for (int j = 0; j < 16; j++) x[j] = px[(16 * (c & 1) + j) * kNttXSi + gc];
        }
        cluster.sync();
        if (fast) {
#pragma unroll
            for (int j = 0; j < 16; j++) xd[j] = __longlong_as_double((long long)x[j]);
            inv_b_d<false>(xd, stwd, 1, c, qd, qinv);
#pragma unroll
            for (int j = 0; j < 16; j++) T[(16 * c + j) * 17 + col] = (u64)__double_as_longlong(xd[j]);
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) xd[j] = __longlong_as_double((long long)T[(c + 16 * j) * 17 + col]);
            inv_a_d<false, false>(xd, stwd, 1, qd, qinv);
            const double nid = (double)c_pc[p].ninv;
            const double2 ni = make_double2(nid, __ddiv_rn(nid, qd));
#pragma unroll
            for (int j = 0; j < 16; j++) {
                double r = mulmod_d(xd[j], ni, qd);  // |r| <= 0.502 q
                if (r < 0.0) r = __dadd_rn(r, qd);
                limb[((size_t)(c + 16 * j) << 8) + gc] =
                    (u64)__double_as_longlong(__dadd_rn(r, 4503599627370496.0)) & 0x000FFFFFFFFFFFFFull;
            }
        } else {
            inv_b(x, W, Wp, 1, c, q);
#pragma unroll
            for (int j = 0; j < 16; j++) T[(16 * c + j) * 17 + col] = x[j];
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; j++) x[j] = T[(c + 16 * j) * 17 + col];
            inv_a(x, W, Wp, 1, q);
            const u64 ni = c_pc[p].ninv, nip = c_pc[p].ninvp;
#pragma unroll
            for (int j = 0; j < 16; j++) limb[((size_t)(c + 16 * j) << 8) + gc] = mul_shoup(x[j], ni, nip, q);
        }
    }
}

// opt-in (HELRM_B200_NTT=cluster): bit-exact, but measured slower than the
// two-pass kernels (B = 128 ciphertexts of 24 limbs: forward 3.61 ms
// against 2.34 ms, inverse 3.92 against 2.54): two 512-thread CTAs per SM
// and two cluster barriers per limb leave too little independent work to
// hide the load and exchange latency
static bool ntt_cluster_on() {
    static int on = -1;
    if (on < 0) {
        const char *e = std::getenv("HELRM_B200_NTT");
        on = (e && std::string(e) == "cluster") ? 1 : 0;
        if (on) {
            cudaFuncSetAttribute(k_ntt_cl<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kNttClWords * 8);
            cudaFuncSetAttribute(k_ntt_cl<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kNttClWords * 8);
        }
    }
    return on == 1;
}

static void ntt256_impl(u64 *data, int nrows, RowMap map, const NttTables &t, bool inv, cudaStream_t s) {
    for (int r0 = 0; r0 < nrows; r0 += 65535) {
        const int nr = nrows - r0 < 65535 ? nrows - r0 : 65535;
        const dim3 grid(16, nr);
        if (ntt_cluster_on()) {
            const dim3 gcl(kNttCl, nr);
            if (!inv)
                k_ntt_cl<false><<<gcl, 512, kNttClWords * 8, s>>>(data, map, t.tw, t.twp, t.twx, t.tws, r0, nullptr,
                                                                  0, 1);
            else
                k_ntt_cl<true><<<gcl, 512, kNttClWords * 8, s>>>(data, map, t.itw, t.itwp, t.itwx, t.itws, r0,
                                                                 nullptr, 0, 1);
            continue;
        }
        if (!inv) {
            k_ntt256_cols<false><<<grid, 256, 0, s>>>(data, map, t.tw, t.twp, t.twx, r0);
            k_ntt256_rows<false><<<grid, 256, 0, s>>>(data, map, t.tw, t.twp, t.twx, t.tws, r0);
        } else {
            k_ntt256_rows<true><<<grid, 256, 0, s>>>(data, map, t.itw, t.itwp, t.itwx, t.itws, r0);
            k_ntt256_cols<true><<<grid, 256, 0, s>>>(data, map, t.itw, t.itwp, t.itwx, r0);
        }
    }
}

static void ntt_impl(u64 *data, int nrows, RowMap map, const NttTables &t, bool inv, cudaStream_t s) {
    if (nrows <= 0) return;
    if (t.logN == 16) {
        int active = nrows;
        if (map.alpha > 0)
            for (int r = 0; r < nrows; r++) active -= map.skip(r) ? 1 : 0;
        const double nwords = (double)active * 65536.0;
        ProfScope ps(inv ? KC_NTT_INV : KC_NTT_FWD, 16.0 * nwords, nwords / 2 * 16, s, 2 * ((nrows + 65534) / 65535));
        ntt256_impl(data, nrows, map, t, inv, s);
        check_launch("ntt256");
        return;
    }
    const int logN = t.logN, logN1 = split_log1(logN), logN2 = logN - logN1;
    const int logC = logN2 < 4 ? logN2 : 4;                    // columns per tile
    int logRB = 12 - logN2;                                     // 4096-word row tiles
    if (logRB < 0) logRB = 0;
    if (logRB > logN1) logRB = logN1;
    const size_t smc = ((size_t)1 << (logN1 + logC)) * sizeof(u64);
    const size_t smr = ((size_t)1 << (logN2 + logRB)) * sizeof(u64);
    static bool attr_done = false;
    if (!attr_done) {
        cudaFuncSetAttribute(k_ntt_cols<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        cudaFuncSetAttribute(k_ntt_cols<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        cudaFuncSetAttribute(k_ntt_rows<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        cudaFuncSetAttribute(k_ntt_rows<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        attr_done = true;
    }
    int active = nrows;
    if (map.alpha > 0)
        for (int r = 0; r < nrows; r++) active -= map.skip(r) ? 1 : 0;
    const double nwords = (double)active * (double)(1 << logN);
    ProfScope ps(inv ? KC_NTT_INV : KC_NTT_FWD, 16.0 * nwords, nwords / 2 * logN, s,
                 2 * ((nrows + 65534) / 65535));
    for (int r0 = 0; r0 < nrows; r0 += 65535) {
        int nr = nrows - r0 < 65535 ? nrows - r0 : 65535;
        dim3 gc(1u << (logN2 - logC), nr), gr(1u << (logN1 - logRB), nr);
        if (!inv) {
            k_ntt_cols<false><<<gc, 256, smc, s>>>(data, map, t.tw, t.twp, logN, logN1, logC, r0);
            k_ntt_rows<false><<<gr, 256, smr, s>>>(data, map, t.tw, t.twp, logN, logN1, logRB, r0);
        } else {
            k_ntt_rows<true><<<gr, 256, smr, s>>>(data, map, t.itw, t.itwp, logN, logN1, logRB, r0);
            k_ntt_cols<true><<<gc, 256, smc, s>>>(data, map, t.itw, t.itwp, logN, logN1, logC, r0);
        }
    }
    check_launch("ntt");
}

// dst[row] = INTT(src row), rows grouped `per_item` to an item of the source
// at src_stride (destination rows contiguous): the first pass reads the
// source, so no copy of the input is made (N = 2^16; other sizes copy first)
void ntt_inverse_from(u64 *dst, const u64 *src, size_t src_stride, int per_item, int nrows, RowMap map,
                      const NttTables &t, cudaStream_t s) {
    if (nrows <= 0) return;
    if (t.logN != 16 || map.alpha > 0) {
        copy_strided(dst, (size_t)per_item << t.logN, src, src_stride, (size_t)per_item << t.logN,
                     nrows / per_item, s);
        ntt_inverse(dst, nrows, map, t, s);
        return;
    }
    if (nrows % per_item) throw std::invalid_argument("ntt_inverse_from: rows not a whole number of items");
    const double nwords = (double)nrows * 65536.0;
    ProfScope ps(KC_NTT_INV, 16.0 * nwords, nwords / 2 * 16, s, 2 * ((nrows + 65534) / 65535));
    for (int r0 = 0; r0 < nrows; r0 += 65535) {
        const int nr = nrows - r0 < 65535 ? nrows - r0 : 65535;
        const dim3 grid(16, nr);
        if (ntt_cluster_on()) {
            k_ntt_cl<true><<<dim3(kNttCl, nr), 512, kNttClWords * 8, s>>>(dst, map, t.itw, t.itwp, t.itwx, t.itws, r0,
                                                                         src, src_stride, per_item);
            continue;
        }
        k_ntt256_rows<true><<<grid, 256, 0, s>>>(dst, map, t.itw, t.itwp, t.itwx, t.itws, r0, src, src_stride,
                                                 per_item);
        k_ntt256_cols<true><<<grid, 256, 0, s>>>(dst, map, t.itw, t.itwp, t.itwx, r0);
    }
    check_launch("ntt256_from");
}

void ntt_forward(u64 *data, int nrows, RowMap map, const NttTables &t, cudaStream_t s) {
    ntt_impl(data, nrows, map, t, false, s);
}
void ntt_inverse(u64 *data, int nrows, RowMap map, const NttTables &t, cudaStream_t s) {
    ntt_impl(data, nrows, map, t, true, s);
}

// =====================================================================
// elementwise
// =====================================================================
struct OpAdd {
    __device__ u64 operator()(u64 a, u64 b, const PrimeConst &pc) const { return add_mod(a, b, pc.q); }
};
struct OpSub {
    __device__ u64 operator()(u64 a, u64 b, const PrimeConst &pc) const { return sub_mod(a, b, pc.q); }
};
struct OpMul {
    __device__ u64 operator()(u64 a, u64 b, const PrimeConst &pc) const { return mul_mod(a, b, pc); }
};

template <class Op>
__global__ void k_ew2(u64 *__restrict__ out, const u64 *__restrict__ a, const u64 *__restrict__ b, size_t npairs,
                      RowMap map, int logN, Op op) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < npairs; i += (size_t)gridDim.x * blockDim.x) {
        const int row = (int)((2 * i) >> logN);
        const PrimeConst &pc = c_pc[map.prime(row)];
        ulonglong2 x = reinterpret_cast<const ulonglong2 *>(a)[i];
        ulonglong2 y = reinterpret_cast<const ulonglong2 *>(b)[i];
        ulonglong2 r;
        r.x = op(x.x, y.x, pc);
        r.y = op(x.y, y.y, pc);
        reinterpret_cast<ulonglong2 *>(out)[i] = r;
    }
}

template <class Op>
static void launch_ew2(u64 *out, const u64 *a, const u64 *b, int nrows, RowMap map, int logN, cudaStream_t s, Op op) {
    size_t npairs = ((size_t)nrows << logN) / 2;
    if (!npairs) return;
    unsigned g = grid1d(npairs, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    ProfScope ps(KC_ELEMENTWISE, 48.0 * npairs, 2.0 * npairs, s, 1);
    k_ew2<Op><<<g, 256, 0, s>>>(out, a, b, npairs, map, logN, op);
    check_launch("elementwise");
}

void ew_add(u64 *out, const u64 *a, const u64 *b, int nrows, RowMap map, int logN, cudaStream_t s) {
    launch_ew2(out, a, b, nrows, map, logN, s, OpAdd());
}
void ew_sub(u64 *out, const u64 *a, const u64 *b, int nrows, RowMap map, int logN, cudaStream_t s) {
    launch_ew2(out, a, b, nrows, map, logN, s, OpSub());
}

__global__ void k_neg(u64 *out, const u64 *a, size_t n, RowMap map, int logN) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int row = (int)(i >> logN);
        out[i] = neg_mod(a[i], c_pc[map.prime(row)].q);
    }
}
void ew_neg(u64 *out, const u64 *a, int nrows, RowMap map, int logN, cudaStream_t s) {
    size_t n = (size_t)nrows << logN;
    unsigned g = grid1d(n, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    ProfScope ps(KC_ELEMENTWISE, 16.0 * n, 0, s, 1);
    k_neg<<<g, 256, 0, s>>>(out, a, n, map, logN);
    check_launch("neg");
}

// out[r] = a[r] mod q(r) for any 64-bit a (Shoup multiplication by 1):
// the import of summed residues from several ranks
__global__ void k_reduce_rows(u64 *out, const u64 *a, size_t n, RowMap map, int logN) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const PrimeConst &pc = c_pc[map.prime((int)(i >> logN))];
        out[i] = mul_shoup(a[i], 1, pc.onep, pc.q);
    }
}
void ew_reduce_rows(u64 *out, const u64 *a, int nrows, RowMap map, int logN, cudaStream_t s) {
    size_t n = (size_t)nrows << logN;
    unsigned g = grid1d(n, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    ProfScope ps(KC_ELEMENTWISE, 16.0 * n, 0, s, 1);
    k_reduce_rows<<<g, 256, 0, s>>>(out, a, n, map, logN);
    check_launch("reduce_rows");
}

// out[pl][i] = a[pl][i] * b[i]
__global__ void k_mul_bcast(u64 *out, const u64 *a, const u64 *b, size_t n, int nq, int logN) {
    const size_t per = (size_t)nq << logN;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t off = i % per;
        const int row = (int)(off >> logN);
        out[i] = mul_mod(a[i], b[off], c_pc[row]);
    }
}
void ew_mul_bcast(u64 *out, const u64 *a, const u64 *b, int npoly, int nq, int, int logN, cudaStream_t s) {
    size_t n = ((size_t)npoly * nq) << logN;
    unsigned g = grid1d(n, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    ProfScope ps(KC_ELEMENTWISE, 8.0 * (2.0 * n + ((double)nq * (1 << logN))), (double)n, s, 1);
    k_mul_bcast<<<g, 256, 0, s>>>(out, a, b, n, nq, logN);
    check_launch("mul_bcast");
}

// the constant's residues travel as a kernel parameter: no device buffer,
// no host copy to wait for
__global__ void k_mul_const(u64 *out, const u64 *a, const ConstWords cw, size_t n, RowMap map, int logN) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int p = map.prime((int)(i >> logN));
        out[i] = mul_shoup(a[i], cw.v[p], cw.vp[p], c_pc[p].q);
    }
}
void ew_mul_const(u64 *out, const u64 *a, const ConstWords &cw, int nrows, RowMap map, int logN, cudaStream_t s) {
    size_t n = (size_t)nrows << logN;
    unsigned g = grid1d(n, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    ProfScope ps(KC_ELEMENTWISE, 16.0 * n, (double)n, s, 1);
    k_mul_const<<<g, 256, 0, s>>>(out, a, cw, n, map, logN);
    check_launch("mul_const");
}

__global__ void k_add_const(u64 *out, const u64 *a, const ConstWords cw, size_t n, RowMap map, int logN) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int p = map.prime((int)(i >> logN));
        out[i] = add_mod(a[i], cw.v[p], c_pc[p].q);
    }
}
void ew_add_const(u64 *out, const u64 *a, const ConstWords &cw, int nrows, RowMap map, int logN, cudaStream_t s) {
    size_t n = (size_t)nrows << logN;
    unsigned g = grid1d(n, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    ProfScope ps(KC_ELEMENTWISE, 16.0 * n, 0, s, 1);
    k_add_const<<<g, 256, 0, s>>>(out, a, cw, n, map, logN);
    check_launch("add_const");
}

__global__ void k_tensor(u64 *out, const u64 *a, const u64 *b, int nq, int logN) {
    const size_t n = (size_t)nq << logN;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const PrimeConst &pc = c_pc[i >> logN];
        u64 a0 = a[i], a1 = a[n + i], b0 = b[i], b1 = b[n + i];
        out[i] = mul_mod(a0, b0, pc);
        u128 acc = {0, 0};
        mac128(acc, a0, b1);
        mac128(acc, a1, b0);
        out[n + i] = reduce128(acc, pc);
        out[2 * n + i] = mul_mod(a1, b1, pc);
    }
}
void ew_tensor(u64 *out, const u64 *a, const u64 *b, int nq, int logN, cudaStream_t s) {
    size_t n = (size_t)nq << logN;
    unsigned g = grid1d(n, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    ProfScope ps(KC_ELEMENTWISE, 56.0 * n, 4.0 * n, s, 1);
    k_tensor<<<g, 256, 0, s>>>(out, a, b, nq, logN);
    check_launch("tensor");
}

__global__ void k_decrypt(u64 *out, const u64 *ct, const u64 *sk, int nq, int logN) {
    const size_t n = (size_t)nq << logN;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const PrimeConst &pc = c_pc[i >> logN];
        out[i] = add_mod(ct[i], mul_mod(ct[n + i], sk[i], pc), pc.q);
    }
}
void ew_decrypt(u64 *out, const u64 *ct, const u64 *sk, int nq, int logN, cudaStream_t s) {
    size_t n = (size_t)nq << logN;
    unsigned g = grid1d(n, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    ProfScope ps(KC_ELEMENTWISE, 32.0 * n, (double)n, s, 1);
    k_decrypt<<<g, 256, 0, s>>>(out, ct, sk, nq, logN);
    check_launch("decrypt");
}

__global__ void k_automorphism(u64 *__restrict__ out, const u64 *__restrict__ in, size_t n, u64 g, int logN) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t rowbase = (i >> logN) << logN;
        const unsigned t = (unsigned)(i - rowbase);
        out[i] = in[rowbase + aut_index(t, g, logN)];
    }
}
void ew_automorphism(u64 *out, const u64 *in, int nrows, u64 galois, int logN, cudaStream_t s) {
    size_t n = (size_t)nrows << logN;
    unsigned g = grid1d(n, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    ProfScope ps(KC_AUTOMORPHISM, 16.0 * n, 0, s, 1);
    k_automorphism<<<g, 256, 0, s>>>(out, in, n, galois, logN);
    check_launch("automorphism");
}

__global__ void k_mac(u64 *out, MacArgs args, int npoly, int nq, int logN) {
    const size_t per = (size_t)nq << logN;
    const size_t n = per * npoly;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t off = i % per;
        const PrimeConst &pc = c_pc[off >> logN];
        u128 acc = {0, 0};
        u64 partial = 0;
        for (int t = 0; t < args.n; t++) {
            mac128(acc, args.ct[t][i], args.pt[t][off]);
            if ((t & 15) == 15) {
                partial = add_mod(partial, reduce128(acc, pc), pc.q);
                acc.lo = acc.hi = 0;
            }
        }
        out[i] = add_mod(partial, reduce128(acc, pc), pc.q);
    }
}
void ew_mac(u64 *out, const MacArgs &args, int npoly, int nq, int logN, cudaStream_t s) {
    size_t n = ((size_t)npoly * nq) << logN;
    unsigned g = grid1d(n, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    const double words = (double)nq * (1 << logN);
    ProfScope ps(KC_ELEMENTWISE, 8.0 * words * (args.n * (npoly + 1) + npoly), words * npoly * args.n, s, 1);
    k_mac<<<g, 256, 0, s>>>(out, args, npoly, nq, logN);
    check_launch("mac");
}

// =====================================================================
// polynomial evaluation: batched degree-1 tensor and the fused linear
// combination every power-basis step and every leaf of the evaluation
// tree reduces to
// =====================================================================
__global__ void k_tensor_batch(u64 *out, const u64 *a, const u64 *b, int nq, int anq, int bnq, size_t as,
                               size_t bs, int logN) {
    const size_t n = (size_t)nq << logN;
    const size_t item = blockIdx.y;
    const u64 *A = a + item * as, *B = b + item * bs;
    const size_t a1 = (size_t)anq << logN, b1 = (size_t)bnq << logN;
    u64 *O = out + item * 3 * n;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const PrimeConst &pc = c_pc[i >> logN];
        const u64 a0 = A[i], x1 = A[a1 + i], b0 = B[i], y1 = B[b1 + i];
        O[i] = mul_mod(a0, b0, pc);
        u128 acc = {0, 0};
        mac128(acc, a0, y1);
        mac128(acc, x1, b0);
        O[n + i] = reduce128(acc, pc);
        O[2 * n + i] = mul_mod(x1, y1, pc);
    }
}
void ew_tensor_batch(u64 *out, const u64 *a, const u64 *b, int nq, int anq, int bnq, int nb, size_t as, size_t bs,
                     int logN, cudaStream_t s) {
    const size_t n = (size_t)nq << logN;
    unsigned g = grid1d(n, 256);
    const unsigned cap = (148u * 64u + nb - 1) / nb;
    if (g > cap) g = cap < 1 ? 1 : cap;
    ProfScope ps(KC_ELEMENTWISE, 56.0 * n * nb, 4.0 * n * nb, s, 1);
    k_tensor_batch<<<dim3(g, nb), 256, 0, s>>>(out, a, b, nq, anq, bnq, as, bs, logN);
    check_launch("tensor_batch");
}

__global__ void k_lincomb(u64 *out, LinCombArgs a, int nq, size_t out_stride, int logN) {
    const size_t per = (size_t)nq << logN;
    const int item = blockIdx.y >> 1, pl = blockIdx.y & 1;
    u64 *O = out + (size_t)item * out_stride + (size_t)pl * per;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < per; i += (size_t)gridDim.x * blockDim.x) {
        const int row = (int)(i >> logN);
        const PrimeConst &pc = c_pc[row];
        u128 acc = {0, 0};
        u64 partial = 0;
        for (int t = 0; t < a.n; t++) {
            const u64 x = a.x[t][(size_t)item * a.xs[t] + ((size_t)pl * a.nq[t] << logN) + i];
            mac128(acc, x, a.coef[(size_t)t * nq + row]);
            if ((t & 15) == 15) {
                partial = add_mod(partial, reduce128(acc, pc), pc.q);
                acc.lo = acc.hi = 0;
            }
        }
        u64 v = add_mod(partial, reduce128(acc, pc), pc.q);
        if (pl == 0 && a.k0) v = add_mod(v, a.k0[row], pc.q);
        O[i] = v;
    }
}
void ew_lincomb(u64 *out, const LinCombArgs &a, int nq, int nb, size_t out_stride, int logN, cudaStream_t s) {
    const size_t per = (size_t)nq << logN;
    unsigned g = grid1d(per, 256);
    const unsigned cap = (148u * 32u + nb - 1) / nb;
    if (g > cap) g = cap < 1 ? 1 : cap;
    ProfScope ps(KC_ELEMENTWISE, 8.0 * per * 2 * nb * (a.n + 1), (double)per * 2 * nb * a.n, s, 1);
    k_lincomb<<<dim3(g, 2 * nb), 256, 0, s>>>(out, a, nq, out_stride, logN);
    check_launch("lincomb");
}

// =====================================================================
// counter-based sampler (SplitMix64 finaliser, Steele-Lea-Flood 2014)
// rand64(seed, domain, idx) = mix(mix(seed ^ mix(domain)) ^ idx); uniform
// residues by Lemire's multiply-shift with rejection (retry counters in
// the top byte of idx); errors centred binomial, eta = 21.
// =====================================================================
__device__ __forceinline__ u64 mix64(u64 z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void k_uniform(u64 *out, size_t n, RowMap map, u64 kseed, u64 idx_base, int logN) {
    const int N = 1 << logN;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int row = (int)(i >> logN);
        const int p = map.prime(row);
        const u64 q = c_pc[p].q;
        const u64 thr = (0ull - q) % q;
        const u64 idx = idx_base + (u64)p * N + (i & (N - 1));
        u64 v = 0;
        for (u64 att = 0; att < 64; att++) {
            u64 r = mix64(kseed ^ (idx + (att << 56)));
            u64 lo = r * q, hi = __umul64hi(r, q);
            if (lo >= thr) { v = hi; break; }
        }
        out[i] = v;
    }
}
void sample_uniform(u64 *out, int nrows, const int *, RowMap map, u64 seed, u64 domain, u64 idx_base, u64,
                    int logN, cudaStream_t s) {
    // host-side part of rand64: mix(seed ^ mix(domain))
    auto hmix = [](u64 z) {
        z += 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    u64 kseed = hmix(seed ^ hmix(domain));
    size_t n = (size_t)nrows << logN;
    unsigned g = grid1d(n, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    ProfScope ps(KC_SAMPLE, 8.0 * n, 0, s, 1);
    k_uniform<<<g, 256, 0, s>>>(out, n, map, kseed, idx_base, logN);
    check_launch("uniform");
}

__global__ void k_cbd(u64 *out, size_t n, RowMap map, u64 kseed, u64 idx_base, int logN) {
    const int N = 1 << logN;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int row = (int)(i >> logN);
        const u64 q = c_pc[map.prime(row)].q;
        u64 r = mix64(kseed ^ (idx_base + (i & (N - 1))));
        int e = __popcll(r & 0x1FFFFFull) - __popcll((r >> 21) & 0x1FFFFFull);
        out[i] = e >= 0 ? (u64)e : q - (u64)(-e);
    }
}
void sample_cbd(u64 *out, int nrows, RowMap map, u64 seed, u64 domain, u64 idx_base, int logN, cudaStream_t s) {
    auto hmix = [](u64 z) {
        z += 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    u64 kseed = hmix(seed ^ hmix(domain));
    size_t n = (size_t)nrows << logN;
    unsigned g = grid1d(n, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    ProfScope ps(KC_SAMPLE, 8.0 * n, 0, s, 1);
    k_cbd<<<g, 256, 0, s>>>(out, n, map, kseed, idx_base, logN);
    check_launch("cbd");
}

__global__ void k_swk_combine(u64 *b, const u64 *a, const u64 *e, const u64 *sk, const u64 *target, const u64 *pmod,
                              size_t n, int lo, int hi, int logN) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int p = (int)(i >> logN);
        const PrimeConst &pc = c_pc[p];
        u64 v = sub_mod(e[i], mul_mod(a[i], sk[i], pc), pc.q);
        if (p >= lo && p < hi) v = add_mod(v, mul_mod(pmod[p], target[i], pc), pc.q);
        b[i] = v;
    }
}
void swk_combine(u64 *b, const u64 *a, const u64 *e, const u64 *sk, const u64 *target, const u64 *pmod, int nrows,
                 int digit_lo, int digit_hi, int logN, cudaStream_t s) {
    size_t n = (size_t)nrows << logN;
    unsigned g = grid1d(n, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    ProfScope ps(KC_SAMPLE, 40.0 * n, 2.0 * n, s, 1);
    k_swk_combine<<<g, 256, 0, s>>>(b, a, e, sk, target, pmod, n, digit_lo, digit_hi, logN);
    check_launch("swk_combine");
}

__global__ void k_enc_combine(u64 *c0, const u64 *a, const u64 *e, const u64 *sk, const u64 *m, size_t n, int logN) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const PrimeConst &pc = c_pc[i >> logN];
        u64 v = sub_mod(e[i], mul_mod(a[i], sk[i], pc), pc.q);
        if (m) v = add_mod(v, m[i], pc.q);
        c0[i] = v;
    }
}
void enc_combine(u64 *c0, const u64 *a, const u64 *e, const u64 *sk, const u64 *m, int nq, int logN, cudaStream_t s) {
    size_t n = (size_t)nq << logN;
    unsigned g = grid1d(n, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    ProfScope ps(KC_SAMPLE, 40.0 * n, (double)n, s, 1);
    k_enc_combine<<<g, 256, 0, s>>>(c0, a, e, sk, m, n, logN);
    check_launch("enc_combine");
}

// =====================================================================
// basis conversion
// =====================================================================
#define HB_MAX_ALPHA 16

// grid: x over N, y over digits j, z over batch.
__global__ void k_modup_bconv(u64 *__restrict__ D, const u64 *__restrict__ X, const u64 *__restrict__ c1ntt,
                              int nq, int K, int L, int alpha, int beta, ModUpTab tab, int logN, size_t in_stride,
                              size_t out_stride, size_t c1_stride) {
    const int N = 1 << logN;
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    const int j = blockIdx.y, b = blockIdx.z;
    const int ne = nq + K;
    const int lo = j * alpha, hi = lo + alpha < nq ? lo + alpha : nq, na = hi - lo;
    const u64 *Xb = X + b * in_stride;
    u64 *Db = D + b * out_stride + (size_t)j * ne * N;
    u64 y[HB_MAX_ALPHA];
    int nneg = 0;
#pragma unroll
    for (int m = 0; m < HB_MAX_ALPHA; m++) {
        if (m < na) {
            const int pm = lo + m;
            const u64 qm = c_pc[pm].q;
            y[m] = mul_shoup(Xb[(size_t)pm * N + n], tab.qhinv[j * alpha + m], tab.qhinvp[j * alpha + m], qm);
            nneg += y[m] > (qm >> 1);
        }
    }
    const u64 *qhat = tab.qhat + (size_t)j * alpha * ne;
    for (int e = 0; e < ne; e++) {
        if (e >= lo && e < hi) {
            Db[(size_t)e * N + n] = c1ntt[b * c1_stride + (size_t)e * N + n];
            continue;
        }
        const int p = e < nq ? e : L + (e - nq);
        const PrimeConst &pc = c_pc[p];
        u128 acc = {0, 0};
#pragma unroll
        for (int m = 0; m < HB_MAX_ALPHA; m++)
            if (m < na) mac128(acc, y[m], qhat[(size_t)m * ne + e]);
        if (nneg) mac128(acc, (u64)nneg, tab.qjneg[(size_t)j * ne + e]);
        Db[(size_t)e * N + n] = reduce128(acc, pc);
    }
}

// The same conversion for primes below 2^60.  q-row targets below 2^40 of a
// digit whose primes are all below 2^40 (digit values y_m below 2^40) on
// the FP64 pipe: exact centred products y_m * qhat_m mod q_e (|t| <= 0.502 q
// each) and the lift term nneg * (-Q_j mod q_e) < 8 q, summed exactly as
// doubles (|S| < 13 q), one reduction per output.  Every other target
// (special primes, wider main primes, or any target of a digit holding a
// wider prime) in split-30 products of two factors below 2^60.  NA = digit
// size, a compile-time constant; blockIdx.y + j0 is the digit.  The digit's
// tables are staged in shared memory.  WIDE = false: every main prime below
// 2^40 (the digits small, every q-row target on the FP64 pipe; the branch
// for the other targets compiled out).
template <int NA, bool WIDE>
__global__ void __launch_bounds__(256)
    k_modup_bconv_split(u64 *__restrict__ D, const u64 *__restrict__ X, const u64 *__restrict__ c1ntt, int nq, int K,
                        int L, int alpha, int j0, ModUpTab tab, int logN, size_t in_stride, size_t out_stride,
                        size_t c1_stride) {
    __shared__ u64 st[(NA + 1) * HB_MAX_PRIMES];      // split-30 qhat [m][e], then qjneg [e]
    __shared__ double2 sd[(NA + 1) * HB_MAX_PRIMES];  // q-row targets: {t, fl(t / q_e)} [m][e], then {qjneg, 0}
    const int N = 1 << logN;
    const int j = j0 + blockIdx.y, b = blockIdx.z;
    const int ne = nq + K;
    const int lo = j * alpha;
    for (int i = threadIdx.x; i < NA * ne; i += blockDim.x) {
        st[i] = tab.qhat_s[(size_t)j * alpha * ne + i];
        sd[i] = tab.qhat_d[(size_t)j * alpha * ne + i];
    }
    for (int i = threadIdx.x; i < ne; i += blockDim.x) {
        st[NA * ne + i] = tab.qjneg_s[(size_t)j * ne + i];
        sd[NA * ne + i] = make_double2(tab.qjneg_d[(size_t)j * ne + i], 0.0);
    }
    __syncthreads();
    // two coefficients per thread, 256 apart: every table value, prime
    // constant and loop step serves two outputs; stores stay coalesced
    const int n0 = blockIdx.x * (2 * blockDim.x) + threadIdx.x;
    if (n0 >= N) return;  // N is a multiple of 512, so n0 + 256 < N as well
    const u64 *Xb = X + b * in_stride;
    u64 *Db = D + b * out_stride + (size_t)j * ne * N;
    u64 y[2][NA];
    double yd[2][NA];
    unsigned nneg[2] = {0, 0};
#pragma unroll
    for (int m = 0; m < NA; m++) {
        const int pm = lo + m;
        const u64 qm = c_pc[pm].q;
        const u64 w = tab.qhinv[j * alpha + m], wp = tab.qhinvp[j * alpha + m];
#pragma unroll
        for (int c = 0; c < 2; c++) {
            const u64 v = mul_shoup(Xb[(size_t)pm * N + n0 + 256 * c], w, wp, qm);
            nneg[c] += v > (qm >> 1);
            y[c][m] = split_pack(v);
            yd[c][m] = u64_to_d(v);
        }
    }
    const double nn0 = u32_to_double(nneg[0]), nn1 = u32_to_double(nneg[1]);
    bool dsmall = true;  // every prime of the digit below 2^40 (block-uniform)
    if (WIDE) {
#pragma unroll
        for (int m = 0; m < NA; m++) dsmall = dsmall && c_pc[lo + m].q < (1ull << 40);
    }
    // q-row targets; the digit's own rows are copies of its input
    for (int e = 0; e < nq; e++) {
        u64 *de = Db + (size_t)e * N + n0;
        if (e >= lo && e < lo + NA) {
            const u64 *ce = c1ntt + b * c1_stride + (size_t)e * N + n0;
            de[0] = ce[0];
            de[256] = ce[256];
            continue;
        }
        const PrimeConst &pc = c_pc[e];
        if (WIDE && (!dsmall || pc.q >= (1ull << 40))) {
            SplitW acc0 = {0, 0, 0}, acc1 = {0, 0, 0};
#pragma unroll
            for (int m = 0; m < NA; m++) {
                const u64 tv = st[m * ne + e];
                splitw_mac(acc0, y[0][m], tv);
                splitw_mac(acc1, y[1][m], tv);
                if ((m & 3) == 3 && m + 1 < NA) {
                    splitw_normalize(acc0);
                    splitw_normalize(acc1);
                }
            }
            const u64 tn = st[NA * ne + e];
            splitw_mac_small(acc0, nneg[0], tn);
            splitw_mac_small(acc1, nneg[1], tn);
            de[0] = dsmall ? splitw_reduce(acc0, pc) : splitw_reduce_wide(acc0, pc);
            de[256] = dsmall ? splitw_reduce(acc1, pc) : splitw_reduce_wide(acc1, pc);
            continue;
        }
        const double qd = u64_to_d(pc.q);
        const double tn = sd[NA * ne + e].x;
        double s0 = __dmul_rn(nn0, tn), s1 = __dmul_rn(nn1, tn);
#pragma unroll
        for (int m = 0; m < NA; m++) {
            const double2 tw = sd[m * ne + e];
            s0 = __dadd_rn(s0, mulmod_d(yd[0][m], tw, qd));
            s1 = __dadd_rn(s1, mulmod_d(yd[1][m], tw, qd));
        }
        de[0] = d_mod_to_u64(s0, qd, pc.qinv);
        de[256] = d_mod_to_u64(s1, qd, pc.qinv);
    }
    // special-prime targets: split-30 products
    for (int e = nq; e < ne; e++) {
        const PrimeConst &pc = c_pc[L + (e - nq)];
        SplitW acc0 = {0, 0, 0}, acc1 = {0, 0, 0};
#pragma unroll
        for (int m = 0; m < NA; m++) {
            const u64 tv = st[m * ne + e];
            splitw_mac(acc0, y[0][m], tv);
            splitw_mac(acc1, y[1][m], tv);
            if ((m & 3) == 3 && m + 1 < NA) {
                splitw_normalize(acc0);
                splitw_normalize(acc1);
            }
        }
        const u64 tn = st[NA * ne + e];
        splitw_mac_small(acc0, nneg[0], tn);
        splitw_mac_small(acc1, nneg[1], tn);
        u64 *de = Db + (size_t)e * N + n0;
        de[0] = dsmall ? splitw_reduce(acc0, pc) : splitw_reduce_wide(acc0, pc);
        de[256] = dsmall ? splitw_reduce(acc1, pc) : splitw_reduce_wide(acc1, pc);
    }
}

template <int NA>
static void modup_split_launch(u64 *D, const u64 *X, const u64 *c1ntt, int nq, int K, int L, int alpha, int j0,
                               int ndig, const ModUpTab &tab, int logN, int nbatch, size_t in_stride,
                               size_t out_stride, size_t c1_stride, cudaStream_t s) {
    dim3 grid(((1 << logN) + 511) / 512, ndig, nbatch);  // two coefficients per thread
    if (tab.split == 2) {
        k_modup_bconv_split<NA, true><<<grid, 256, 0, s>>>(D, X, c1ntt, nq, K, L, alpha, j0, tab, logN, in_stride,
                                                           out_stride, c1_stride);
        return;
    }
    k_modup_bconv_split<NA, false><<<grid, 256, 0, s>>>(D, X, c1ntt, nq, K, L, alpha, j0, tab, logN, in_stride, out_stride,
                                                  c1_stride);
}
static void modup_split_dispatch(int na, u64 *D, const u64 *X, const u64 *c1ntt, int nq, int K, int L, int alpha,
                                 int j0, int ndig, const ModUpTab &tab, int logN, int nbatch, size_t in_stride,
                                 size_t out_stride, size_t c1_stride, cudaStream_t s) {
#define HB_MU_CASE(A)                                                                                             \
    case A:                                                                                                        \
        modup_split_launch<A>(D, X, c1ntt, nq, K, L, alpha, j0, ndig, tab, logN, nbatch, in_stride, out_stride,    \
                              c1_stride, s);                                                                       \
        break;
    switch (na) {
        HB_MU_CASE(1) HB_MU_CASE(2) HB_MU_CASE(3) HB_MU_CASE(4) HB_MU_CASE(5) HB_MU_CASE(6) HB_MU_CASE(7)
        HB_MU_CASE(8)
        default: throw std::invalid_argument("modup_bconv: split digit size out of range");
    }
#undef HB_MU_CASE
}

void modup_bconv(u64 *D, const u64 *X, const u64 *c1ntt, int nq, int K, int L, int alpha, int beta,
                  const ModUpTab &tab, int logN, int nbatch, size_t in_stride, size_t out_stride, size_t c1_stride,
                  cudaStream_t s) {
    if (alpha > HB_MAX_ALPHA) throw std::invalid_argument("alpha exceeds HB_MAX_ALPHA");
    const int N = 1 << logN;
    const int ne = nq + K;
    if (ne > HB_MAX_PRIMES) throw std::invalid_argument("modup_bconv: too many primes");
    ProfScope ps(KC_MODUP_BCONV, 8.0 * nbatch * (double)N * (nq + (double)beta * ne),
                 (double)nbatch * N * ((double)nq + (double)alpha * ((double)beta * ne - nq)), s, 1);
    if (tab.split && alpha <= 8 && N >= 512) {
        const int full = nq / alpha, rag = nq - full * alpha;
        if (full > 0)
            modup_split_dispatch(alpha, D, X, c1ntt, nq, K, L, alpha, 0, full, tab, logN, nbatch, in_stride,
                                 out_stride, c1_stride, s);
        if (rag > 0)
            modup_split_dispatch(rag, D, X, c1ntt, nq, K, L, alpha, full, 1, tab, logN, nbatch, in_stride,
                                 out_stride, c1_stride, s);
    } else {
        dim3 grid((N + 255) / 256, beta, nbatch);
        k_modup_bconv<<<grid, 256, 0, s>>>(D, X, c1ntt, nq, K, L, alpha, beta, tab, logN, in_stride, out_stride,
                                           c1_stride);
    }
    check_launch("modup_bconv");
}

__global__ void k_moddown_bconv(u64 *__restrict__ Z, const u64 *__restrict__ Y, int nq, int K, int L, ModDownTab tab,
                                int logN, size_t in_stride, size_t out_stride) {
    const int N = 1 << logN;
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    const int b = blockIdx.y;
    const u64 *Yb = Y + b * in_stride;
    u64 *Zb = Z + b * out_stride;
    u64 y[8];
    int nneg = 0;
#pragma unroll
    for (int k = 0; k < 8; k++)
        if (k < K) {
            const u64 pk = c_pc[L + k].q;
            y[k] = mul_shoup(Yb[(size_t)k * N + n], tab.phinv[k], tab.phinvp[k], pk);
            nneg += y[k] > (pk >> 1);
        }
    for (int i = 0; i < nq; i++) {
        u128 acc = {0, 0};
#pragma unroll
        for (int k = 0; k < 8; k++)
            if (k < K) mac128(acc, y[k], tab.phat[(size_t)k * nq + i]);
        if (nneg) mac128(acc, (u64)nneg, tab.pneg[i]);
        Zb[(size_t)i * N + n] = reduce128(acc, c_pc[i]);
    }
}
// The same conversion with split-30 products (every prime below 2^60: table
// entries and special-prime values below 2^60).  KK = number of special
// primes; the phat and pneg rows are staged in shared memory.
template <int KK>
__global__ void __launch_bounds__(256)
    k_moddown_bconv_split(u64 *__restrict__ Z, const u64 *__restrict__ Y, int nq, int L, ModDownTab tab, int logN,
                          size_t in_stride, size_t out_stride) {
    __shared__ u64 st[(KK + 1) * HB_MAX_PRIMES];  // phat [k][i], then pneg [i]
    for (int i = threadIdx.x; i < KK * nq; i += blockDim.x) st[i] = tab.phat_s[i];
    for (int i = threadIdx.x; i < nq; i += blockDim.x) st[KK * nq + i] = tab.pneg_s[i];
    __syncthreads();
    // two coefficients per thread, 256 apart (N is a multiple of 512): every
    // table value and loop step serves two outputs; stores stay coalesced
    const int N = 1 << logN;
    const int n0 = blockIdx.x * 512 + threadIdx.x;
    const int b = blockIdx.y;
    const u64 *Yb = Y + b * in_stride;
    u64 *Zb = Z + b * out_stride;
    u64 y[2][KK];
    unsigned nneg[2] = {0, 0};
#pragma unroll
    for (int k = 0; k < KK; k++) {
        const u64 pk = c_pc[L + k].q;
#pragma unroll
        for (int c = 0; c < 2; c++) {
            const u64 v = mul_shoup(Yb[(size_t)k * N + n0 + 256 * c], tab.phinv[k], tab.phinvp[k], pk);
            nneg[c] += v > (pk >> 1);
            y[c][k] = split_pack(v);
        }
    }
    for (int i = 0; i < nq; i++) {
        SplitW a0 = {0, 0, 0}, a1 = {0, 0, 0};
#pragma unroll
        for (int k = 0; k < KK; k++) {
            const u64 tv = st[k * nq + i];
            splitw_mac(a0, tv, y[0][k]);
            splitw_mac(a1, tv, y[1][k]);
            if ((k & 3) == 3 && k + 1 < KK) {
                splitw_normalize(a0);
                splitw_normalize(a1);
            }
        }
        const u64 tn = st[KK * nq + i];
        splitw_mac_small(a0, nneg[0], tn);
        splitw_mac_small(a1, nneg[1], tn);
        const PrimeConst &pc = c_pc[i];
        // table entries below 2^40 keep every partial sum in the narrow
        // reduction's range
        const bool narrow = pc.q < (1ull << 40);
        Zb[(size_t)i * N + n0] = narrow ? splitw_reduce(a0, pc) : splitw_reduce_wide(a0, pc);
        Zb[(size_t)i * N + n0 + 256] = narrow ? splitw_reduce(a1, pc) : splitw_reduce_wide(a1, pc);
    }
}

void moddown_bconv(u64 *Z, const u64 *Y, int nq, int K, int L, const ModDownTab &tab, int logN, int nbatch,
                   size_t in_stride, size_t out_stride, cudaStream_t s) {
    if (K > 8) throw std::invalid_argument("at most 8 special primes");
    if (nq > HB_MAX_PRIMES) throw std::invalid_argument("moddown_bconv: too many primes");
    const int N = 1 << logN;
    dim3 grid((N + 255) / 256, nbatch);
    const dim3 grid2(N / 512, nbatch);  // the split kernel: two coefficients per thread
    ProfScope ps(KC_MODDOWN_BCONV, 8.0 * nbatch * (double)N * (K + nq), (double)nbatch * N * (K + (double)K * nq), s,
                 1);
    if (tab.split && N >= 512) {
        switch (K) {
#define HB_MD_CASE(A)                                                                                             \
    case A:                                                                                                        \
        k_moddown_bconv_split<A><<<grid2, 256, 0, s>>>(Z, Y, nq, L, tab, logN, in_stride, out_stride);             \
        break;
            HB_MD_CASE(1) HB_MD_CASE(2) HB_MD_CASE(3) HB_MD_CASE(4) HB_MD_CASE(5) HB_MD_CASE(6) HB_MD_CASE(7)
            HB_MD_CASE(8)
#undef HB_MD_CASE
            default:
                k_moddown_bconv<<<grid, 256, 0, s>>>(Z, Y, nq, K, L, tab, logN, in_stride, out_stride);
        }
    } else {
        k_moddown_bconv<<<grid, 256, 0, s>>>(Z, Y, nq, K, L, tab, logN, in_stride, out_stride);
    }
    check_launch("moddown_bconv");
}

__global__ void k_moddown_combine(u64 *out, const u64 *x, const u64 *Z, int nq, ModDownTab tab, const u64 *addend,
                                  u64 g, int logN, size_t x_stride, size_t z_stride, size_t out_stride,
                                  size_t add_stride, const u64 *add2, size_t add2_stride) {
    const int N = 1 << logN;
    const size_t n = (size_t)nq << logN;
    const int b = blockIdx.y;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int row = (int)(i >> logN);
        const u64 q = c_pc[row].q;
        u64 v = mul_shoup(sub_mod(x[b * x_stride + i], Z[b * z_stride + i], q), tab.pinv[row], tab.pinvp[row], q);
        if (addend) {
            const unsigned t = (unsigned)(i & (N - 1));
            const unsigned src = g == 1 ? t : aut_index(t, g, logN);
            v = add_mod(v, addend[b * add_stride + ((size_t)row << logN) + src], q);
        }
        if (add2) v = add_mod(v, add2[b * add2_stride + i], q);
        out[b * out_stride + i] = v;
    }
}
void moddown_combine(u64 *out, const u64 *x, const u64 *Z, int nq, const ModDownTab &tab, const u64 *addend,
                     u64 add_galois, int logN, int nbatch, size_t x_stride, size_t z_stride, size_t out_stride,
                     size_t add_stride, cudaStream_t s, const u64 *add2, size_t add2_stride) {
    size_t n = (size_t)nq << logN;
    unsigned g = grid1d(n, 256);
    if (g > 4096) g = 4096;
    dim3 grid(g, nbatch);
    ProfScope ps(KC_MODDOWN_COMBINE, 8.0 * nbatch * (double)n * (3 + (addend ? 1 : 0) + (add2 ? 1 : 0)),
                 (double)nbatch * n, s, 1);
    k_moddown_combine<<<grid, 256, 0, s>>>(out, x, Z, nq, tab, addend, add_galois, logN, x_stride, z_stride,
                                           out_stride, add_stride, add2, add2_stride);
    check_launch("moddown_combine");
}

// =====================================================================
// rescale
// =====================================================================
__global__ void k_rescale_prep(u64 *W, const u64 *R, int npoly, int nq_out, u64 ql, int logN, size_t r_stride,
                               size_t w_stride) {
    const size_t n = ((size_t)npoly * nq_out) << logN;
    const int N = 1 << logN;
    const int b = blockIdx.y;
    const u64 h = ql >> 1;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int rowall = (int)(i >> logN);
        const int pl = rowall / nq_out, row = rowall % nq_out;
        const PrimeConst &pc = c_pc[row];
        u64 r = R[b * r_stride + (size_t)pl * N + (i & (N - 1))];
        r = add_mod(r, h, ql);
        u64 rq = mul_shoup(r, 1ull, pc.onep, pc.q);
        u64 hq = mul_shoup(h, 1ull, pc.onep, pc.q);
        W[b * w_stride + i] = sub_mod(hq, rq, pc.q);
    }
}
void rescale_prep(u64 *W, const u64 *R, int npoly, int nq_out, u64 ql, int logN, int nbatch, size_t r_stride,
                  size_t w_stride, cudaStream_t s) {
    size_t n = ((size_t)npoly * nq_out) << logN;
    unsigned g = grid1d(n, 256);
    if (g > 4096) g = 4096;
    ProfScope ps(KC_RESCALE, 8.0 * nbatch * ((double)n + (double)((size_t)npoly << logN)), 0, s, 1);
    k_rescale_prep<<<dim3(g, nbatch), 256, 0, s>>>(W, R, npoly, nq_out, ql, logN, r_stride, w_stride);
    check_launch("rescale_prep");
}

__global__ void k_rescale_combine(u64 *out, const u64 *c, const u64 *W, int npoly, int nq_in, const u64 *qlinv,
                                  const u64 *qlinvp, int logN, size_t c_stride, size_t w_stride, size_t out_stride) {
    const int nq_out = nq_in - 1;
    const size_t n = ((size_t)npoly * nq_out) << logN;
    const int N = 1 << logN;
    const int b = blockIdx.y;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int rowall = (int)(i >> logN);
        const int pl = rowall / nq_out, row = rowall % nq_out;
        const u64 q = c_pc[row].q;
        const u64 cv = c[b * c_stride + ((size_t)pl * nq_in + row) * N + (i & (N - 1))];
        out[b * out_stride + i] = mul_shoup(add_mod(cv, W[b * w_stride + i], q), qlinv[row], qlinvp[row], q);
    }
}
void rescale_combine(u64 *out, const u64 *c, const u64 *W, int npoly, int nq_in, const u64 *qlinv, const u64 *qlinvp,
                     int logN, int nbatch, size_t c_stride, size_t w_stride, size_t out_stride, cudaStream_t s) {
    size_t n = ((size_t)npoly * (nq_in - 1)) << logN;
    unsigned g = grid1d(n, 256);
    if (g > 4096) g = 4096;
    ProfScope ps(KC_RESCALE, 24.0 * nbatch * (double)n, (double)nbatch * n, s, 1);
    k_rescale_combine<<<dim3(g, nbatch), 256, 0, s>>>(out, c, W, npoly, nq_in, qlinv, qlinvp, logN, c_stride,
                                                      w_stride, out_stride);
    check_launch("rescale_combine");
}

// =====================================================================
// key switching: key multiplication with the automorphism folded into the
// digit gather.
// =====================================================================
// One thread block per (ciphertext, 256 coefficients of one limb row), the
// ciphertext index fastest: the blocks that read the same key segment run
// back to back, so each key segment comes from DRAM once per launch and from
// L2 for the other ciphertexts.  Limbs below 2^40 use Karatsuba split-29
// products, the others 128-bit products.  This form serves digit counts
// other than four; four digits run the batch-looping forms below
// (k_keymult_loop for one giant step, k_keymult_group for several).
#ifndef HB_KEYMULT_BLOCKS
#define HB_KEYMULT_BLOCKS 6  // resident blocks per SM (occupancy hides the gathers' latency)
#endif
// BETA > 0: the digit count as a compile-time constant (registers for
// exactly BETA digits); BETA = 0: read at run time (up to HB_MAX_BETA)
template <int BETA>
__global__ void __launch_bounds__(256, HB_KEYMULT_BLOCKS) k_keymult(u64 *__restrict__ acc, const u64 *__restrict__ D,
                                                 const u64 *__restrict__ key, u64 g, int nq, int K, int L, int beta_rt,
                                                 int keyP, const u64 *__restrict__ addb, int accumulate, int logN,
                                                 size_t d_stride, size_t acc_stride, size_t add_stride) {
    constexpr int MB = BETA ? BETA : HB_MAX_BETA;
    const int beta = BETA ? BETA : beta_rt;
    const int N = 1 << logN;
    const int ne = nq + K;
    const size_t n_all = (size_t)ne << logN;
    const int b = blockIdx.x;
    const size_t i = (size_t)blockIdx.y * 256 + threadIdx.x;
    if (i >= n_all) return;
    const u64 *Db = D + b * d_stride;
    u64 *Ab = acc + b * acc_stride;
    const int e = (int)(i >> logN);
    const unsigned t = (unsigned)(i & (N - 1));
    const unsigned src = g == 1 ? t : aut_index(t, g, logN);
    const int p = e < nq ? e : L + (e - nq);
    const PrimeConst &pc = c_pc[p];
    // issue every digit gather and key load before the products; base
    // pointers and strides once, one add per digit
    const u64 *dp = Db + ((size_t)e << logN) + src;
    const size_t dstep = n_all;
    const u64 *kp = key + ((size_t)p << logN) + t;
    const size_t kstep = (size_t)keyP << logN;
    u64 dv[MB], kbv[MB], kav[MB];
#pragma unroll
    for (int j = 0; j < MB; j++)
        if (j < beta) {
            dv[j] = dp[j * dstep];
            kbv[j] = kp[(2 * j) * kstep];
            kav[j] = kp[(2 * j + 1) * kstep];
        }
    u64 vb, va;
    if (pc.q < (1ull << 40)) {
        Kara29 sb = {0, 0, 0}, sa = {0, 0, 0};
#pragma unroll
        for (int j = 0; j < MB; j++)
            if (j < beta) {
                const u64 d = k29_pack(dv[j]);
                const unsigned ds = k29_sum(d);
                k29_mac(sb, k29_pack(kbv[j]), d, ds);
                k29_mac(sa, k29_pack(kav[j]), d, ds);
            }
        vb = k29_reduce(sb, pc);
        va = k29_reduce(sa, pc);
    } else {
        u128 sb = {0, 0}, sa = {0, 0};
#pragma unroll
        for (int j = 0; j < MB; j++)
            if (j < beta) {
                mac128(sb, dv[j], kbv[j]);
                mac128(sa, dv[j], kav[j]);
            }
        vb = reduce128(sb, pc);
        va = reduce128(sa, pc);
    }
    if (addb) vb = add_mod(vb, addb[b * add_stride + ((size_t)e << logN) + src], pc.q);
    if (accumulate) {
        vb = add_mod(vb, Ab[i], pc.q);
        va = add_mod(va, Ab[n_all + i], pc.q);
    }
    Ab[i] = vb;
    Ab[n_all + i] = va;
}
// The batch-looping form (four digits): one thread per coefficient of one
// limb row, looping over the ciphertexts of the batch.  The key words of
// the coefficient (split-29 halves and their sums on limbs below 2^40) and
// the automorphism index stay in registers across the batch, so per
// ciphertext a thread only gathers its digits and the addend and updates
// the accumulator.
#ifndef HB_KEYMULT_LOOP_BLOCKS
#define HB_KEYMULT_LOOP_BLOCKS 4
#endif
template <int BETA>
__global__ void __launch_bounds__(256, HB_KEYMULT_LOOP_BLOCKS)
    k_keymult_loop(u64 *__restrict__ acc, const u64 *__restrict__ D, const u64 *__restrict__ key, u64 g, int nq,
                   int K, int L, int keyP, const u64 *__restrict__ addb, int accumulate, int logN, int nbatch,
                   size_t d_stride, size_t acc_stride, size_t add_stride) {
    const int ne = nq + K;
    const size_t n_all = (size_t)ne << logN;
    const int e = blockIdx.y;
    const unsigned t = blockIdx.x * 256u + threadIdx.x;
    const unsigned src = g == 1 ? t : aut_index(t, g, logN);
    const int p = e < nq ? e : L + (e - nq);
    const PrimeConst pc = c_pc[p];
    const u64 *kp = key + ((size_t)p << logN) + t;
    const size_t kstep = (size_t)keyP << logN;
    const size_t drow = ((size_t)e << logN) + src, irow = ((size_t)e << logN) + t;
    if (pc.q < (1ull << 40)) {
        unsigned kbl[BETA], kbh[BETA], kbs[BETA], kal[BETA], kah[BETA], kas[BETA];
#pragma unroll
        for (int j = 0; j < BETA; j++) {
            const u64 kb = k29_pack(kp[(2 * j) * kstep]), ka = k29_pack(kp[(2 * j + 1) * kstep]);
            kbl[j] = (unsigned)kb, kbh[j] = (unsigned)(kb >> 32), kbs[j] = kbl[j] + kbh[j];
            kal[j] = (unsigned)ka, kah[j] = (unsigned)(ka >> 32), kas[j] = kal[j] + kah[j];
        }
#pragma unroll 2
        for (int b = 0; b < nbatch; b++) {
            const u64 *dp = D + b * d_stride + drow;
            u64 dv[BETA];
#pragma unroll
            for (int j = 0; j < BETA; j++) dv[j] = dp[j * n_all];
            Kara29 sb = {0, 0, 0}, sa = {0, 0, 0};
#pragma unroll
            for (int j = 0; j < BETA; j++) {
                const u64 d = k29_pack(dv[j]);
                const unsigned dl = (unsigned)d, dh = (unsigned)(d >> 32), ds = dl + dh;
                k29_mac_s(sb, kbl[j], kbh[j], kbs[j], dl, dh, ds);
                k29_mac_s(sa, kal[j], kah[j], kas[j], dl, dh, ds);
            }
            u64 vb = k29_reduce(sb, pc), va = k29_reduce(sa, pc);
            if (addb) vb = add_mod(vb, addb[b * add_stride + drow], pc.q);
            u64 *A = acc + b * acc_stride + irow;
            if (accumulate) {
                vb = add_mod(vb, A[0], pc.q);
                va = add_mod(va, A[n_all], pc.q);
            }
            A[0] = vb;
            A[n_all] = va;
        }
    } else {
        u64 kb[BETA], ka[BETA];
#pragma unroll
        for (int j = 0; j < BETA; j++) {
            kb[j] = kp[(2 * j) * kstep];
            ka[j] = kp[(2 * j + 1) * kstep];
        }
        for (int b = 0; b < nbatch; b++) {
            const u64 *dp = D + b * d_stride + drow;
            u128 sb = {0, 0}, sa = {0, 0};
#pragma unroll
            for (int j = 0; j < BETA; j++) {
                const u64 d = dp[j * n_all];
                mac128(sb, d, kb[j]);
                mac128(sa, d, ka[j]);
            }
            u64 vb = reduce128(sb, pc), va = reduce128(sa, pc);
            if (addb) vb = add_mod(vb, addb[b * add_stride + drow], pc.q);
            u64 *A = acc + b * acc_stride + irow;
            if (accumulate) {
                vb = add_mod(vb, A[0], pc.q);
                va = add_mod(va, A[n_all], pc.q);
            }
            A[0] = vb;
            A[n_all] = va;
        }
    }
}

// G giant steps in one pass (four digits each): acc += sum_i KS(D_i, key_i)
// + sigma_i(addb_i).  The accumulator is read and written once for all G,
// and the 8G products of each output share one reduction (split-29 sums
// hold up to 33 terms; 128-bit sums of 8G 120-bit products stay below
// 2^125 for G <= 4).  The key words of every giant stay in registers.
struct GiantSet {
    const u64 *D[HB_MAX_GIANTS], *key[HB_MAX_GIANTS], *addb[HB_MAX_GIANTS];
    u64 g[HB_MAX_GIANTS];
};
template <int G>
__global__ void __launch_bounds__(256, G <= 2 ? 3 : 2)
    k_keymult_group(u64 *__restrict__ acc, GiantSet gs, int nq, int K, int L, int keyP, int accumulate, int logN,
                    int nbatch, size_t d_stride, size_t acc_stride, size_t add_stride) {
    constexpr int B = 4;
    const int ne = nq + K;
    const size_t n_all = (size_t)ne << logN;
    const int e = blockIdx.y;
    const unsigned t = blockIdx.x * 256u + threadIdx.x;
    const int p = e < nq ? e : L + (e - nq);
    const PrimeConst pc = c_pc[p];
    const size_t kofs = ((size_t)p << logN) + t, kstep = (size_t)keyP << logN;
    const size_t erow = (size_t)e << logN, irow = erow + t;
    size_t drow[G];
#pragma unroll
    for (int gi = 0; gi < G; gi++) drow[gi] = erow + (gs.g[gi] == 1 ? t : aut_index(t, gs.g[gi], logN));
    if (pc.q < (1ull << 40)) {
        unsigned kl[G][2][B], kh[G][2][B], ks[G][2][B];  // [giant][b/a][digit]
#pragma unroll
        for (int gi = 0; gi < G; gi++)
#pragma unroll
            for (int j = 0; j < B; j++)
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const u64 k = k29_pack(gs.key[gi][kofs + (2 * j + c) * kstep]);
                    kl[gi][c][j] = (unsigned)k, kh[gi][c][j] = (unsigned)(k >> 32);
                    ks[gi][c][j] = kl[gi][c][j] + kh[gi][c][j];
                }
        for (int b = 0; b < nbatch; b++) {
            Kara29 sb = {0, 0, 0}, sa = {0, 0, 0};
            u64 vb = 0;
#pragma unroll
            for (int gi = 0; gi < G; gi++) {
                const u64 *dp = gs.D[gi] + b * d_stride + drow[gi];
                u64 dv[B];
#pragma unroll
                for (int j = 0; j < B; j++) dv[j] = dp[j * n_all];
#pragma unroll
                for (int j = 0; j < B; j++) {
                    const u64 d = k29_pack(dv[j]);
                    const unsigned dl = (unsigned)d, dh = (unsigned)(d >> 32), ds = dl + dh;
                    k29_mac_s(sb, kl[gi][0][j], kh[gi][0][j], ks[gi][0][j], dl, dh, ds);
                    k29_mac_s(sa, kl[gi][1][j], kh[gi][1][j], ks[gi][1][j], dl, dh, ds);
                }
                vb = add_mod(vb, gs.addb[gi][b * add_stride + drow[gi]], pc.q);
            }
            vb = add_mod(vb, k29_reduce(sb, pc), pc.q);
            u64 va = k29_reduce(sa, pc);
            u64 *A = acc + b * acc_stride + irow;
            if (accumulate) {
                vb = add_mod(vb, A[0], pc.q);
                va = add_mod(va, A[n_all], pc.q);
            }
            A[0] = vb;
            A[n_all] = va;
        }
    } else {
        for (int b = 0; b < nbatch; b++) {
            u128 sb = {0, 0}, sa = {0, 0};
            u64 vb = 0;
#pragma unroll
            for (int gi = 0; gi < G; gi++) {
                const u64 *dp = gs.D[gi] + b * d_stride + drow[gi];
                const u64 *kp = gs.key[gi] + kofs;
#pragma unroll
                for (int j = 0; j < B; j++) {
                    const u64 d = dp[j * n_all];
                    mac128(sb, d, kp[(2 * j) * kstep]);
                    mac128(sa, d, kp[(2 * j + 1) * kstep]);
                }
                vb = add_mod(vb, gs.addb[gi][b * add_stride + drow[gi]], pc.q);
            }
            vb = add_mod(vb, reduce128(sb, pc), pc.q);
            u64 va = reduce128(sa, pc);
            u64 *A = acc + b * acc_stride + irow;
            if (accumulate) {
                vb = add_mod(vb, A[0], pc.q);
                va = add_mod(va, A[n_all], pc.q);
            }
            A[0] = vb;
            A[n_all] = va;
        }
    }
}

void keymult_group(u64 *acc, int ngiants, const u64 *const *D, const u64 *const *keys, const u64 *galois,
                   const u64 *const *addb, int nq, int K, int L, int beta, int keyP, bool accumulate, int logN,
                   int nbatch, size_t d_stride, size_t acc_stride, size_t add_stride, cudaStream_t s) {
    if (beta != 4 || logN < 8 || nq + K > 65535 || ngiants < 2 || ngiants > HB_MAX_GIANTS)
        throw std::invalid_argument("keymult_group: four digits, 2..HB_MAX_GIANTS giants, N >= 256");
    GiantSet gs{};
    for (int i = 0; i < ngiants; i++) {
        gs.D[i] = D[i];
        gs.key[i] = keys[i];
        gs.addb[i] = addb[i];
        gs.g[i] = galois[i];
    }
    const double nd = (double)((size_t)(nq + K) << logN);
    ProfScope ps(KC_KEYMULT,
                 8.0 * (nbatch * nd * (ngiants * (beta + 1.0) + (accumulate ? 4.0 : 2.0)) + 2.0 * ngiants * beta * nd),
                 2.0 * ngiants * beta * nbatch * nd, s, 1);
    const dim3 grid(1u << (logN - 8), nq + K);
    const int acc_i = accumulate ? 1 : 0;
    switch (ngiants) {
        case 2: k_keymult_group<2><<<grid, 256, 0, s>>>(acc, gs, nq, K, L, keyP, acc_i, logN, nbatch, d_stride, acc_stride, add_stride); break;
        case 3: k_keymult_group<3><<<grid, 256, 0, s>>>(acc, gs, nq, K, L, keyP, acc_i, logN, nbatch, d_stride, acc_stride, add_stride); break;
        default: k_keymult_group<4><<<grid, 256, 0, s>>>(acc, gs, nq, K, L, keyP, acc_i, logN, nbatch, d_stride, acc_stride, add_stride); break;
    }
    check_launch("keymult_group");
}

void keymult(u64 *acc, const u64 *D, const u64 *key, u64 galois, int nq, int K, int L, int beta, int keyP,
             const u64 *addb, bool accumulate, int logN, int nbatch, size_t d_stride, size_t acc_stride,
             size_t add_stride, cudaStream_t s) {
    if (beta > HB_MAX_BETA) throw std::invalid_argument("keymult: more digits than HB_MAX_BETA");
    size_t n = (size_t)(nq + K) << logN;
    const size_t chunks = (n + 255) / 256;
    if (chunks > 65535) throw std::invalid_argument("keymult: limb stack too large for one launch");
    // digits per ciphertext + the key once per launch + accumulator traffic
    const double nd = (double)n;
    ProfScope ps(KC_KEYMULT,
                 8.0 * (nbatch * nd * (beta + 2.0 + (addb ? 1.0 : 0.0) + (accumulate ? 2.0 : 0.0)) + 2.0 * beta * nd),
                 2.0 * beta * nbatch * nd, s, 1);
    if (beta == 4 && logN >= 8 && nq + K <= 65535) {
        k_keymult_loop<4><<<dim3(1u << (logN - 8), nq + K), 256, 0, s>>>(
            acc, D, key, galois, nq, K, L, keyP, addb, accumulate ? 1 : 0, logN, nbatch, d_stride, acc_stride,
            add_stride);
        check_launch("keymult_loop");
        return;
    }
    const dim3 grid(nbatch, (unsigned)chunks);
#define HB_KM_ARGS acc, D, key, galois, nq, K, L, beta, keyP, addb, accumulate ? 1 : 0, logN, d_stride, acc_stride, add_stride
    switch (beta) {
        case 1: k_keymult<1><<<grid, 256, 0, s>>>(HB_KM_ARGS); break;
        case 2: k_keymult<2><<<grid, 256, 0, s>>>(HB_KM_ARGS); break;
        case 3: k_keymult<3><<<grid, 256, 0, s>>>(HB_KM_ARGS); break;
        case 4: k_keymult<4><<<grid, 256, 0, s>>>(HB_KM_ARGS); break;
        default: k_keymult<0><<<grid, 256, 0, s>>>(HB_KM_ARGS); break;
    }
#undef HB_KM_ARGS
    check_launch("keymult");
}

// =====================================================================
// fused baby steps + diagonal MAC (double hoisting): see hb_bsgs.cuh
// =====================================================================
// Every instantiation of the fused MAC may take up to the per-block limit
// of dynamic shared memory: set once for all of them (a launch allocates
// only what it asks for).  Two launchers with their own high-water marks
// would lower each other's settings.
static void bsgs_mac_attributes() {
    static bool done = false;
    if (done) return;
    const int lim = 227 * 1024;
    cudaFuncSetAttribute(k_bsgs_mac<HB_BCH, 4, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(k_bsgs_mac<0, 4, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(k_bsgs_mac<HB_BCH, 4, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(k_bsgs_mac<0, 4, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(k_bsgs_mac<HB_BCH, 0, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(k_bsgs_mac<0, 0, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(k_bsgs_mac<HB_BCH, 4, 1, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(k_bsgs_mac<HB_BCH, 4, 2, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(k_bsgs_mac<HB_BCH, 2, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(k_bsgs_mac<HB_BCH, 3, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(k_bsgs_mac<HB_BCH, 4, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(k_bsgs_mac<HB_BCH, 5, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(k_bsgs_mac<HB_BCH, 6, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(k_bsgs_mac<HB_BCH, 7, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    done = true;
}

void bsgs_baby_mac(u64 *inner, const u64 *ct, const u64 *D, const BsgsChunk &ch, int nq, int K, int L, int beta,
                   int keyP, int pt_nq, const u64 *pmod_q, int logN, int nbatch, size_t ct_stride, size_t d_stride,
                   size_t inner_stride, cudaStream_t s) {
    if (ch.nbabies > HB_BCH || ch.gcount > HB_GCH) throw std::invalid_argument("bsgs chunk too large");
    const bool split = beta == 4 && primes_sized(0, nq, true) && primes_sized(L, K, false);
    const bool full = ch.nbabies == HB_BCH;
    // chunks of at most half the giant slots: two batch items per iteration
    const bool pair = split && full && ch.gcount <= HB_GCH / 2 && nbatch > 1;
    // full chunks of 2 to 7 digits over mixed rows (primes on both sides of
    // 2^40, e.g. a 50-bit q0 or 60-bit bootstrapping primes): the fixed-shape
    // kernel with the product form chosen per row.  Not one digit: the
    // fixed shape runs the identity baby as a rotated one whose key tile
    // holds P at digit 0 (for c0) and digit 1 (for c1)
    const bool fixed_mixed = !split && full && beta >= 2 && beta <= 7;
    const size_t smem = bsgs_smem_words(beta, pair ? 2 : 1, (split && full) || fixed_mixed) * 8;
    if (smem > 227 * 1024 || beta > HB_MAX_BETA)
        throw std::invalid_argument("bsgs: too many digits for the shared-memory key tile");
    bsgs_mac_attributes();
    const size_t n = (size_t)(nq + K) << logN;
    // per ciphertext: c0/c1 rows, the digits, the inner sums written; per
    // launch: every baby key and plaintext of the chunk once
    const double nd = (double)n, nqw = (double)nq * (1 << logN);
    ProfScope ps(KC_BSGS_MAC,
                 8.0 * (nbatch * (2.0 * nqw + beta * nd + 2.0 * ch.gcount * nd * (ch.accumulate ? 2 : 1)) +
                        2.0 * beta * ch.nkeys * nd + ch.npts * nd),
                 (double)nbatch * nd * (2.0 * beta * ch.nkeys + 2.0 * ch.npts), s, split && K ? 2 : 1);
    // specialised for full chunks, four digits (the dnum-4 key of the
    // benchmark parameter sets at the top level) and q rows below 2^40 with
    // special rows above it: one launch per kind of row, each with a single
    // product form.  Anything else runs the generic form over every row.
#define HB_BSGS_LAUNCH(NBF_, BETA_, ROWS_, PAIR_, E0_, NROWS_)                                                  \
    k_bsgs_mac<NBF_, BETA_, ROWS_, PAIR_><<<dim3((1u << logN) / HB_BT, NROWS_), HB_GCH * HB_BT, smem, s>>>(    \
        inner, ct, D, ch, nq, K, L, beta, keyP, pt_nq, pmod_q, logN, nbatch, E0_, ct_stride, d_stride, inner_stride)
    if (split) {
        if (pair) {
            HB_BSGS_LAUNCH(HB_BCH, 4, 1, 2, 0, nq);
            if (K) HB_BSGS_LAUNCH(HB_BCH, 4, 2, 2, nq, K);
        } else if (full) {
            HB_BSGS_LAUNCH(HB_BCH, 4, 1, 1, 0, nq);
            if (K) HB_BSGS_LAUNCH(HB_BCH, 4, 2, 1, nq, K);
        } else {
            HB_BSGS_LAUNCH(0, 4, 1, 1, 0, nq);
            if (K) HB_BSGS_LAUNCH(0, 4, 2, 1, nq, K);
        }
    } else if (fixed_mixed) {
        if (beta == 2) HB_BSGS_LAUNCH(HB_BCH, 2, 0, 1, 0, nq + K);
        else if (beta == 3) HB_BSGS_LAUNCH(HB_BCH, 3, 0, 1, 0, nq + K);
        else if (beta == 4) HB_BSGS_LAUNCH(HB_BCH, 4, 0, 1, 0, nq + K);
        else if (beta == 5) HB_BSGS_LAUNCH(HB_BCH, 5, 0, 1, 0, nq + K);
        else if (beta == 6) HB_BSGS_LAUNCH(HB_BCH, 6, 0, 1, 0, nq + K);
        else HB_BSGS_LAUNCH(HB_BCH, 7, 0, 1, 0, nq + K);
    } else {
        if (full) HB_BSGS_LAUNCH(HB_BCH, 0, 0, 1, 0, nq + K);
        else HB_BSGS_LAUNCH(0, 0, 0, 1, 0, nq + K);
    }
#undef HB_BSGS_LAUNCH
    check_launch("bsgs_mac");
}

// ---- one-pass plaintext x ciphertext matrix products (the IVE lookup) ------------
// out_r = sum_k T[r][k] * ct_k for a rows x cols table T of broadcast
// constants (one word per prime) or of plaintext polynomials, every input
// ciphertext read once for all rows of the launch (the reference's
// ConstMatMulKernel / PlaintextMatMulKernel, cheddar_pybind.cu:1044-1569).
// One thread per coefficient position of one (poly, limb) row; RB rows
// accumulated as exact centred FP64 remainders (each below 0.502 q < 2^35.1
// for q < 2^40, so up to 2^17 terms sum exactly) and reduced once.
constexpr int kMmKT = 64;  // table columns staged per shared-memory tile

template <int RB, bool PT>
__global__ void __launch_bounds__(256) k_table_matmul(MatMulArgs a) {
    __shared__ double2 s_c[RB * kMmKT];          // constants as {c, fl(c/q)}
    __shared__ const u64 *s_p[RB * kMmKT];       // or plaintext limb pointers
    __shared__ const u64 *s_x[kMmKT];            // input ciphertext rows
    const int N = 1 << a.logN;
    const int rowid = blockIdx.y;                // poly * nq + limb
    const int pl = rowid / a.nq, e = rowid - pl * a.nq;
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const PrimeConst pc = c_pc[e];
    const double qd = u64_to_d(pc.q);
    double acc[RB];
#pragma unroll
    for (int r = 0; r < RB; r++) acc[r] = 0.0;
    const int rows = min(RB, a.rows - a.r0);
    for (int k0 = 0; k0 < a.cols; k0 += kMmKT) {
        const int kt = min(kMmKT, a.cols - k0);
        __syncthreads();
        for (int t = threadIdx.x; t < RB * kt; t += blockDim.x) {
            const int r = t / kt, kk = t - r * kt;
            if (PT) {
                s_p[r * kMmKT + kk] = r < rows ? a.pts[(size_t)(a.r0 + r) * a.cols + k0 + kk] + ((size_t)e << a.logN)
                                               : nullptr;
            } else {
                const double c = r < rows ? a.tab[((size_t)e * a.rows + a.r0 + r) * a.cols + k0 + kk] : 0.0;
                s_c[r * kMmKT + kk] = make_double2(c, __dmul_rn(c, pc.qinv));
            }
        }
        for (int t = threadIdx.x; t < kt; t += blockDim.x)
            s_x[t] = a.x[(size_t)(k0 + t) * 2 + pl] + ((size_t)e << a.logN);
        __syncthreads();
        if (n < N) {
            for (int kk = 0; kk < kt; kk++) {
                const double y = u64_to_d(__ldcs(s_x[kk] + n));
#pragma unroll
                for (int r = 0; r < RB; r++) {
                    if (PT) {
                        if (r < rows) {
                            const double w = u64_to_d(__ldg(s_p[r * kMmKT + kk] + n));
                            acc[r] = __dadd_rn(acc[r], mulmod_d(y, make_double2(w, __dmul_rn(w, pc.qinv)), qd));
                        }
                    } else {
                        acc[r] = __dadd_rn(acc[r], mulmod_d(y, s_c[r * kMmKT + kk], qd));
                    }
                }
            }
        }
    }
    if (n < N) {
#pragma unroll
        for (int r = 0; r < RB; r++)
            if (r < rows) a.out[a.r0 + r][((size_t)rowid << a.logN) + n] = d_mod_to_u64(acc[r], qd, pc.qinv);
    }
}

void table_matmul(const MatMulArgs &args, bool pt, cudaStream_t s) {
    if (args.cols <= 0 || args.rows <= 0 || args.cols > (1 << 16))
        throw std::invalid_argument("table_matmul: bad table shape");
    for (int i = 0; i < args.nq; i++)
        if (g_host_q[i] >= (1ull << 40)) throw std::invalid_argument("table_matmul: primes of 40 bits and more");
    const int N = 1 << args.logN;
    const double words = (double)args.nq * N;
    for (int r0 = 0; r0 < args.rows; r0 += 16) {
        MatMulArgs a = args;
        a.r0 = r0;
        const int rb = std::min(16, args.rows - r0);
        // per pass: every input ciphertext once, the rows written once, and
        // the plaintexts (a plaintext table) once
        ProfScope ps(KC_ELEMENTWISE,
                     8.0 * words * (2.0 * args.cols + 2.0 * rb + (pt ? (double)rb * args.cols : 0.0)),
                     2.0 * words * rb * args.cols, s, 1);
        const dim3 grid((N + 255) / 256, 2 * args.nq);
#define HB_MM(RB_)                                                                 \
    (pt ? (void)k_table_matmul<RB_, true><<<grid, 256, 0, s>>>(a)                   \
        : (void)k_table_matmul<RB_, false><<<grid, 256, 0, s>>>(a))
        if (rb == 1) HB_MM(1);
        else if (rb <= 4) HB_MM(4);
        else HB_MM(16);
#undef HB_MM
        check_launch("table_matmul");
    }
}

// ---- the tensor-core MAC (hb_bsgs_tc.cuh) ------------------------------------
bool bsgs_mma_supported(int nq, int beta) {
    if (beta < 1 || beta > 4 || nq < 1 || nq > g_host_nq) return false;
    for (int i = 0; i < nq; i++)
        if (g_host_q[i] >= (1ull << 37)) return false;
    return true;
}
size_t bsgs_mma_planes_bytes(int nq, int logN) { return (size_t)nq * ((size_t)1 << logN) / kTcCoef * kTcPtTile; }

void bsgs_mma_planes(uint8_t *ptp, const BsgsChunk &ch, int nq, int logN, cudaStream_t s) {
    if (ch.nbabies > 32 || ch.gcount > HB_GCH) throw std::invalid_argument("bsgs_mma: chunk too large");
    ProfScope ps(KC_ELEMENTWISE, (double)nq * (1 << logN) * (8.0 * ch.npts / ch.gcount + kTcPlanes * 512.0 / kTcCoef),
                 0.0, s, 1);
    const int N = 1 << logN;
    k_pt_planes<<<dim3((N + 127) / 128, nq), 128, 0, s>>>(ptp, ch.babies, ch.nbabies, ch.gcount, logN);
    check_launch("pt_planes");
}

void bsgs_mma_class_consts(u64 *out, const u64 *primes, int nq) {
    for (int e = 0; e < nq; e++) {
        const unsigned __int128 q = primes[e];
        unsigned __int128 v = 1;
        for (int c = 0; c < kTcClasses; c++) {
            out[(size_t)e * kTcClasses + c] = (u64)(v % q);
            v = (v % q) << 8;
        }
    }
}

void bsgs_baby_mma(u64 *inner, const u64 *ct, const u64 *D, const BsgsChunk &ch, const u64 *cls, int nq, int K,
                   int L, int beta, int keyP, const u64 *pmod_q, int logN, int nbatch, size_t ct_stride,
                   size_t d_stride, size_t inner_stride, int *err, cudaStream_t s) {
    (void)L;
    if (!ch.ptp || ch.nbabies > 32 || ch.gcount > HB_GCH || !bsgs_mma_supported(nq, beta))
        throw std::invalid_argument("bsgs_mma: unsupported chunk or primes");
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(k_bsgs_mma<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
        cudaFuncSetAttribute(k_bsgs_mma<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
        cudaFuncSetAttribute(k_bsgs_mma<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
        cudaFuncSetAttribute(k_bsgs_mma<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
        attr = true;
    }
    static int nsm = 0;
    if (!nsm) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
        if (nsm <= 0) nsm = 148;
    }
    const long tiles = (long)nq * ((1 << logN) / kTcCoef);
    const int grid = (int)std::min<long>(nsm, tiles);
    const double nqw = (double)nq * (1 << logN);
    // a pass waits on nothing outside itself; 2 s bounds every pipeline wait
    const unsigned long long limit_ns = 2000000000ull;
    for (int ct0 = 0; ct0 < nbatch; ct0 += kTcCts) {
        const int nb = std::min(kTcCts, nbatch - ct0);
        // per pass: the chunk's keys (q rows) and plaintext planes once; per
        // ciphertext: the q rows of c0/c1 and of the digits, the inner sums written
        ProfScope ps(KC_BSGS_MMA,
                     nb * 8.0 * (2.0 * nqw + beta * nqw + 2.0 * ch.gcount * nqw * (ch.accumulate ? 2 : 1)) +
                         8.0 * 2.0 * beta * ch.nkeys * nqw + (double)bsgs_mma_planes_bytes(nq, logN),
                     (double)nb * nqw * (2.0 * beta * ch.nkeys + 2.0 * ch.npts), s, 1);
#define HB_MMA_LAUNCH(B_)                                                                                       \
    k_bsgs_mma<B_><<<grid, kTcThreads, kTcSmem, s>>>(inner, ct, D, ch, ch.ptp, cls, nq, K, keyP, pmod_q, logN,   \
                                                     nbatch, ct0, ct_stride, d_stride, inner_stride, err, limit_ns)
        switch (beta) {
            case 1: HB_MMA_LAUNCH(1); break;
            case 2: HB_MMA_LAUNCH(2); break;
            case 3: HB_MMA_LAUNCH(3); break;
            default: HB_MMA_LAUNCH(4); break;
        }
#undef HB_MMA_LAUNCH
        check_launch("bsgs_mma");
    }
}

void bsgs_baby_mac_special(u64 *inner, const u64 *ct, const u64 *D, const BsgsChunk &ch, int nq, int K, int L,
                           int beta, int keyP, int pt_nq, const u64 *pmod_q, int logN, int nbatch,
                           size_t ct_stride, size_t d_stride, size_t inner_stride, cudaStream_t s) {
    if (K == 0) return;
    if (ch.nbabies > HB_BCH || ch.gcount > HB_GCH) throw std::invalid_argument("bsgs chunk too large");
    const size_t smem = bsgs_smem_words(beta) * 8;
    if (smem > 227 * 1024 || beta > HB_MAX_BETA)
        throw std::invalid_argument("bsgs: too many digits for the shared-memory key tile");
    bsgs_mac_attributes();
    const double kd = (double)K * (1 << logN);
    ProfScope ps(KC_BSGS_MAC,
                 8.0 * (nbatch * (beta * kd + 2.0 * ch.gcount * kd * (ch.accumulate ? 2 : 1)) +
                        2.0 * beta * ch.nkeys * kd + ch.npts * kd),
                 (double)nbatch * kd * (2.0 * beta * ch.nkeys + 2.0 * ch.npts), s, 1);
    const bool split = beta == 4 && primes_sized(L, K, false);
    const int e0 = nq;
    if (split && ch.nbabies == HB_BCH)
        k_bsgs_mac<HB_BCH, 4, 2><<<dim3((1u << logN) / HB_BT, K), HB_GCH * HB_BT, smem, s>>>(
            inner, ct, D, ch, nq, K, L, beta, keyP, pt_nq, pmod_q, logN, nbatch, e0, ct_stride, d_stride,
            inner_stride);
    else if (split)
        k_bsgs_mac<0, 4, 2><<<dim3((1u << logN) / HB_BT, K), HB_GCH * HB_BT, smem, s>>>(
            inner, ct, D, ch, nq, K, L, beta, keyP, pt_nq, pmod_q, logN, nbatch, e0, ct_stride, d_stride,
            inner_stride);
    else
        k_bsgs_mac<0, 0, 0><<<dim3((1u << logN) / HB_BT, K), HB_GCH * HB_BT, smem, s>>>(
            inner, ct, D, ch, nq, K, L, beta, keyP, pt_nq, pmod_q, logN, nbatch, e0, ct_stride, d_stride,
            inner_stride);
    check_launch("bsgs_mac_special");
}

// ---- batched copies ----------------------------------------------------------
__global__ void k_copy_strided(ulonglong2 *__restrict__ dst, size_t dstride2, const ulonglong2 *__restrict__ src,
                               size_t sstride2, size_t n2) {
    const size_t b = blockIdx.y;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n2; i += (size_t)gridDim.x * blockDim.x)
        dst[b * dstride2 + i] = src[b * sstride2 + i];
}
__global__ void k_gather_items(ulonglong2 *__restrict__ dst, PtrBatch seg0, PtrBatch seg1, int nseg, size_t n2) {
    const int b = blockIdx.y;
    for (int j = 0; j < nseg; j++) {
        const ulonglong2 *src = reinterpret_cast<const ulonglong2 *>(j == 0 ? seg0.p[b] : seg1.p[b]);
        ulonglong2 *d = dst + ((size_t)b * nseg + j) * n2;
        for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n2; i += (size_t)gridDim.x * blockDim.x)
            d[i] = src[i];
    }
}
__global__ void k_scatter_items(PtrBatchW dst, const ulonglong2 *__restrict__ src, size_t n2) {
    const int b = blockIdx.y;
    ulonglong2 *d = reinterpret_cast<ulonglong2 *>(dst.p[b]);
    const ulonglong2 *sb = src + (size_t)b * n2;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n2; i += (size_t)gridDim.x * blockDim.x)
        d[i] = sb[i];
}
static void copy_check(size_t words, int nb) {
    if (words % 2 || nb <= 0 || nb > 65535) throw std::invalid_argument("batched copy: bad shape");
}
static unsigned copy_grid(size_t n2) {
    size_t g = (n2 + 255) / 256;
    return (unsigned)(g > 1024 ? 1024 : g);
}
void copy_strided(u64 *dst, size_t dstride, const u64 *src, size_t sstride, size_t words, int nb, cudaStream_t s) {
    copy_check(words, nb);
    if (dstride % 2 || sstride % 2) throw std::invalid_argument("copy_strided: odd stride");
    ProfScope ps(KC_ELEMENTWISE, 16.0 * words * nb, 0.0, s, 1);
    k_copy_strided<<<dim3(copy_grid(words / 2), nb), 256, 0, s>>>(
        reinterpret_cast<ulonglong2 *>(dst), dstride / 2, reinterpret_cast<const ulonglong2 *>(src), sstride / 2,
        words / 2);
    check_launch("copy_strided");
}
void gather_items(u64 *dst, const PtrBatch &seg0, const PtrBatch &seg1, int nseg, size_t words, int nb,
                  cudaStream_t s) {
    copy_check(words, nb);
    if (nb > HB_PTR_BATCH || nseg < 1 || nseg > 2) throw std::invalid_argument("gather_items: bad batch");
    ProfScope ps(KC_ELEMENTWISE, 16.0 * words * nb * nseg, 0.0, s, 1);
    k_gather_items<<<dim3(copy_grid(words / 2), nb), 256, 0, s>>>(reinterpret_cast<ulonglong2 *>(dst), seg0, seg1,
                                                                   nseg, words / 2);
    check_launch("gather_items");
}
void scatter_items(const PtrBatchW &dst, const u64 *src, size_t words, int nb, cudaStream_t s) {
    copy_check(words, nb);
    if (nb > HB_PTR_BATCH) throw std::invalid_argument("scatter_items: bad batch");
    ProfScope ps(KC_ELEMENTWISE, 16.0 * words * nb, 0.0, s, 1);
    k_scatter_items<<<dim3(copy_grid(words / 2), nb), 256, 0, s>>>(dst, reinterpret_cast<const ulonglong2 *>(src),
                                                                    words / 2);
    check_launch("scatter_items");
}

// =====================================================================
// device CKKS encoding (the upload side of the path)
// With n = N/2 slots and zeta = exp(i pi / N), slot j is m(zeta^(5^j mod 2N)).
// Writing m(X) = sum_{k<n} (m_k + X^n m_{k+n}) X^k and using zeta^(g n) = i for
// g = 1 mod 4, the slots are the length-n DFT of w_k zeta^k (w_k = m_k + i
// m_{k+n}) at position r = (5^j mod 2N - 1) / 4.  Encoding inverts that:
// place slot j at r_j, take the unnormalised inverse DFT y, then
// w_k = zeta^-k y_k / n and m_k = round(scale Re w_k), m_{k+n} = round(scale
// Im w_k).  The DFT is radix-2 decimation in time in FP64: the input is
// scattered straight into bit-reversed order, the first log2(min(n, 2048))
// stages run on contiguous 2048-point blocks in shared memory, the remaining
// ones on strided columns of 2048 points, also in shared memory.
// =====================================================================
namespace {
constexpr int kEncBlock = 2048;  // complex points per block (32 KB of shared memory)

__device__ __forceinline__ double2 cmul(double2 a, double2 b) {
    return make_double2(__fma_rn(a.x, b.x, -a.y * b.y), __fma_rn(a.x, b.y, a.y * b.x));
}
}  // namespace

__global__ void k_enc_tables(int *perm, double2 *tw, int logN) {
    const unsigned n = 1u << (logN - 1);
    const u64 m2 = 2ull << logN;
    for (unsigned j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) {
        u64 g = 1, b = 5, e = j;
        while (e) {
            if (e & 1) g = g * b % m2;
            b = b * b % m2;
            e >>= 1;
        }
        const unsigned r = (unsigned)((g - 1) >> 2);
        perm[j] = (int)(__brev(r) >> (33 - logN));
        if (j < n / 2) {
            double sn, cs;
            sincospi(2.0 * (double)j / (double)n, &sn, &cs);
            tw[j] = make_double2(cs, -sn);  // exp(-2 pi i j / n)
        }
    }
}
void enc_tables(int *perm, double2 *tw, int logN, cudaStream_t s) {
    const unsigned n = 1u << (logN - 1);
    k_enc_tables<<<grid1d(n, 256), 256, 0, s>>>(perm, tw, logN);
    check_launch("enc_tables");
}

__global__ void k_enc_scatter(double2 *z, const double *vals, int nvals, int cplx, const int *perm, int h) {
    const unsigned n = 1u << h;
    const size_t v = blockIdx.y;
    for (unsigned j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) {
        double2 x = make_double2(0.0, 0.0);
        if ((int)j < nvals) {
            const double *src = vals + v * (size_t)nvals * (cplx ? 2 : 1);
            x = cplx ? make_double2(src[2 * j], src[2 * j + 1]) : make_double2(src[j], 0.0);
        }
        z[v * n + perm[j]] = x;
    }
}
void enc_scatter(double2 *z, const double *vals, int nvals, int cplx, int count, const EncTables &t, cudaStream_t s) {
    const unsigned n = 1u << (t.logN - 1);
    ProfScope ps(KC_ELEMENTWISE, (double)count * n * (cplx ? 32.0 : 24.0), 0.0, s, 1);
    k_enc_scatter<<<dim3(grid1d(n, 256), count), 256, 0, s>>>(z, vals, nvals, cplx, t.perm, t.logN - 1);
    check_launch("enc_scatter");
}

// stages 0 .. cs-1 on contiguous blocks of 2^cs points
__global__ void __launch_bounds__(kEncBlock / 2) k_enc_fft_rows(double2 *z, const double2 *tw, int h, int cs) {
    __shared__ double2 a[kEncBlock];
    const unsigned n = 1u << h, C = 1u << cs;
    double2 *blk = z + (size_t)blockIdx.y * n + (size_t)blockIdx.x * C;
    for (unsigned i = threadIdx.x; i < C; i += blockDim.x) a[i] = blk[i];
    __syncthreads();
    for (int st = 0; st < cs; st++) {
        const unsigned half = 1u << st;
        for (unsigned p = threadIdx.x; p < C / 2; p += blockDim.x) {
            const unsigned k = p & (half - 1), i0 = ((p >> st) << (st + 1)) + k, i1 = i0 + half;
            const double2 w = tw[(size_t)k * (n >> (st + 1))];
            const double2 u = a[i0], t = cmul(w, a[i1]);
            a[i0] = make_double2(u.x + t.x, u.y + t.y);
            a[i1] = make_double2(u.x - t.x, u.y - t.y);
        }
        __syncthreads();
    }
    for (unsigned i = threadIdx.x; i < C; i += blockDim.x) blk[i] = a[i];
}

// stages cs .. h-1 on blocks of bc consecutive columns x 2^(h-cs) rows
__global__ void __launch_bounds__(kEncBlock / 2) k_enc_fft_cols(double2 *z, const double2 *tw, int h, int cs) {
    __shared__ double2 a[kEncBlock];
    const unsigned n = 1u << h, C = 1u << cs, R = n >> cs, bc = kEncBlock / R;
    const unsigned b0 = blockIdx.x * bc;
    double2 *vec = z + (size_t)blockIdx.y * n;
    for (unsigned i = threadIdx.x; i < kEncBlock; i += blockDim.x) {
        const unsigned j = i / bc, c = i % bc;
        a[i] = vec[(size_t)j * C + b0 + c];
    }
    __syncthreads();
    for (int st = cs; st < h; st++) {
        const int sp = st - cs;
        const unsigned half = 1u << sp;
        for (unsigned p = threadIdx.x; p < kEncBlock / 2; p += blockDim.x) {
            const unsigned c = p % bc, jp = p / bc;
            const unsigned kk = jp & (half - 1), j0 = ((jp >> sp) << (sp + 1)) + kk, j1 = j0 + half;
            const unsigned k = b0 + c + kk * C;  // index inside the span of 2^(st+1)
            const double2 w = tw[(size_t)k * (n >> (st + 1))];
            const double2 u = a[j0 * bc + c], t = cmul(w, a[j1 * bc + c]);
            a[j0 * bc + c] = make_double2(u.x + t.x, u.y + t.y);
            a[j1 * bc + c] = make_double2(u.x - t.x, u.y - t.y);
        }
        __syncthreads();
    }
    for (unsigned i = threadIdx.x; i < kEncBlock; i += blockDim.x) {
        const unsigned j = i / bc, c = i % bc;
        vec[(size_t)j * C + b0 + c] = a[i];
    }
}

void enc_ifft(double2 *z, int count, const EncTables &t, cudaStream_t s) {
    const int h = t.logN - 1;
    const unsigned n = 1u << h;
    const int cs = h < 11 ? h : 11;
    const unsigned C = 1u << cs;
    ProfScope ps(KC_ELEMENTWISE, (double)count * n * 32.0 * (h > cs ? 2 : 1), 0.0, s, h > cs ? 2 : 1);
    k_enc_fft_rows<<<dim3(n / C, count), C / 2 > 1 ? C / 2 : 1, 0, s>>>(z, t.tw, h, cs);
    check_launch("enc_fft_rows");
    if (h > cs) {
        const unsigned R = n >> cs;
        if (R > (unsigned)kEncBlock) throw std::invalid_argument("enc_ifft: ring too large");
        k_enc_fft_cols<<<dim3(C / (kEncBlock / R), count), kEncBlock / 2, 0, s>>>(z, t.tw, h, cs);
        check_launch("enc_fft_cols");
    }
}

__global__ void k_enc_round(PtrBatchW dst, const double2 *z, int rows, RowMap map, double scale, int logN) {
    const unsigned N = 1u << logN, n = N >> 1;
    const size_t v = blockIdx.y;
    u64 *out = dst.p[v];
    const double inv_n = 1.0 / (double)n;
    for (unsigned k = blockIdx.x * blockDim.x + threadIdx.x; k < n; k += gridDim.x * blockDim.x) {
        const double2 y = z[v * n + k];
        double sn, cs;
        sincospi((double)k / (double)N, &sn, &cs);  // zeta^-k = cs - i sn
        const double re = (y.x * cs + y.y * sn) * inv_n * scale;
        const double im = (y.y * cs - y.x * sn) * inv_n * scale;
        const long long a = __double2ll_rn(re), b = __double2ll_rn(im);
        const u64 ua = (u64)(a < 0 ? -a : a), ub = (u64)(b < 0 ? -b : b);
        for (int r = 0; r < rows; r++) {
            const PrimeConst &pc = c_pc[map.prime(r)];
            const u64 ma = mul_shoup(ua, 1ull, pc.onep, pc.q), mb = mul_shoup(ub, 1ull, pc.onep, pc.q);
            out[(size_t)r * N + k] = (a < 0 && ma) ? pc.q - ma : ma;
            out[(size_t)r * N + k + n] = (b < 0 && mb) ? pc.q - mb : mb;
        }
    }
}
void enc_round(const PtrBatchW &dst, const double2 *z, int rows, RowMap map, double scale, int count,
               const EncTables &t, cudaStream_t s) {
    if (count > HB_PTR_BATCH) throw std::invalid_argument("enc_round: bad batch");
    const unsigned n = 1u << (t.logN - 1);
    ProfScope ps(KC_ELEMENTWISE, (double)count * n * (16.0 + 16.0 * rows), 0.0, s, 1);
    k_enc_round<<<dim3(grid1d(n, 256), count), 256, 0, s>>>(dst, z, rows, map, scale, t.logN);
    check_launch("enc_round");
}

// ---- decoding on the device: the inverse of the encoding above ---------------
// Coefficients from the first nc limbs (after the inverse NTT) by Garner's
// mixed radix, centred as the host CRT did (digits compared with
// (q_k - 1) / 2 from the top; a value above (Q - 1) / 2 is recomputed from
// the negated residues), evaluated in FP64 by Horner from the top digit and
// divided by the scale.  Then y_k = (m_k + i m_{k+n}) zeta^k and the slots
// are the length-n DFT with exp(+2 pi i r k / n) at r_j: the encoding's FFT
// (exp(-2 pi i ...), bit-reversed input) on conj(y), conjugated back.
__global__ void k_dec_crt(double *out, const u64 *limbs, DecCrt c, double inv_scale, int logN) {
    const unsigned N = 1u << logN;
    for (unsigned t = blockIdx.x * blockDim.x + threadIdx.x; t < N; t += gridDim.x * blockDim.x) {
        u64 r[HB_DEC_MAX], d[HB_DEC_MAX];
        for (int i = 0; i < c.n; i++) r[i] = limbs[((size_t)i << logN) + t];
        bool neg = false;
        for (int pass = 0; pass < 2; pass++) {
            if (pass) {
                for (int i = 0; i < c.n; i++) r[i] = r[i] ? c_pc[i].q - r[i] : 0;
            }
            for (int i = 0; i < c.n; i++) {
                const PrimeConst &pc = c_pc[i];
                u64 acc = 0;
                for (int k = 0; k < i; k++) acc = add_mod(acc, mul_mod(d[k], c.mmod[i * HB_DEC_MAX + k], pc), pc.q);
                d[i] = mul_mod(sub_mod(r[i], acc, pc.q), c.minv[i], pc);
            }
            if (pass) break;
            bool gt = false;
            for (int i = c.n - 1; i >= 0; i--) {
                const u64 h = (c_pc[i].q - 1) / 2;
                if (d[i] != h) {
                    gt = d[i] > h;
                    break;
                }
            }
            if (!gt) break;
            neg = true;
        }
        double v = 0.0;
        for (int i = c.n - 1; i >= 0; i--) v = __fma_rn(v, (double)c_pc[i].q, (double)d[i]);
        out[t] = (neg ? -v : v) * inv_scale;
    }
}
__global__ void k_dec_twist(double2 *z, const double *m, int logN) {
    const unsigned N = 1u << logN, n = N >> 1;
    const int h = logN - 1;
    for (unsigned k = blockIdx.x * blockDim.x + threadIdx.x; k < n; k += gridDim.x * blockDim.x) {
        double sn, cs;
        sincospi((double)k / (double)N, &sn, &cs);  // zeta^k = cs + i sn
        const double a = m[k], b = m[k + n];
        z[__brev(k) >> (32 - h)] = make_double2(a * cs - b * sn, -(a * sn + b * cs));  // conj(y_k)
    }
}
__global__ void k_dec_gather(double *out, const double2 *z, const int *perm, int cplx, int h) {
    const unsigned n = 1u << h;
    for (unsigned j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) {
        const double2 v = z[__brev((unsigned)perm[j]) >> (32 - h)];  // r_j
        if (cplx) {
            out[2 * j] = v.x;
            out[2 * j + 1] = -v.y;
        } else {
            out[j] = v.x;
        }
    }
}
void decode_slots(double *out, const u64 *limbs, const DecCrt &c, double scale, int cplx, double *coef, double2 *z,
                  const EncTables &t, cudaStream_t s) {
    if (c.n < 1 || c.n > HB_DEC_MAX) throw std::invalid_argument("decode: 1 to 4 limbs");
    const unsigned N = 1u << t.logN, n = N >> 1;
    {
        ProfScope ps(KC_ELEMENTWISE, (double)N * (8.0 * c.n + 16.0) + (double)n * 16.0, 0.0, s, 2);
        k_dec_crt<<<grid1d(N, 256), 256, 0, s>>>(coef, limbs, c, 1.0 / scale, t.logN);
        check_launch("dec_crt");
        k_dec_twist<<<grid1d(n, 256), 256, 0, s>>>(z, coef, t.logN);
        check_launch("dec_twist");
    }
    enc_ifft(z, 1, t, s);
    ProfScope ps(KC_ELEMENTWISE, (double)n * (16.0 + 4.0 + 8.0 * (cplx ? 2 : 1)), 0.0, s, 1);
    k_dec_gather<<<grid1d(n, 256), 256, 0, s>>>(out, z, t.perm, cplx, t.logN - 1);
    check_launch("dec_gather");
}

// slot-wise multiplication by i (X^(N/2)) and the conjugation lane split
__global__ void k_mul_iunit(u64 *out, const u64 *in, int nrows, int nq, const u64 *iu, int logN) {
    const size_t n = (size_t)nrows << logN;
    const unsigned half = 1u << (logN - 1), mask = (1u << logN) - 1;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int p = (int)(i >> logN) % nq;
        const int sel = ((unsigned)i & mask) >= half ? 2 : 0;
        out[i] = mul_shoup(in[i], iu[4 * p + sel], iu[4 * p + sel + 1], c_pc[p].q);
    }
}
void ew_mul_iunit(u64 *out, const u64 *in, int nrows, int nq, const u64 *iu, int logN, cudaStream_t s) {
    const size_t n = (size_t)nrows << logN;
    unsigned g = grid1d(n, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    ProfScope ps(KC_ELEMENTWISE, 16.0 * n, (double)n, s, 1);
    k_mul_iunit<<<g, 256, 0, s>>>(out, in, nrows, nq, iu, logN);
    check_launch("mul_iunit");
}

__global__ void k_lane_split(PtrBatchW ev, PtrBatchW od, const u64 *pk, const u64 *cj, int nq, const u64 *iu,
                             int logN) {
    const size_t n = (size_t)(2 * nq) << logN;
    const size_t base = blockIdx.y * n;
    u64 *E = ev.p[blockIdx.y], *O = od.p[blockIdx.y];
    const unsigned half = 1u << (logN - 1), mask = (1u << logN) - 1;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int p = (int)(i >> logN) % nq;
        const u64 q = c_pc[p].q;
        const u64 a = pk[base + i], b = cj[base + i];
        const int sel = ((unsigned)i & mask) >= half ? 2 : 0;
        E[i] = add_mod(a, b, q);
        O[i] = mul_shoup(sub_mod(b, a, q), iu[4 * p + sel], iu[4 * p + sel + 1], q);
    }
}
void lane_split(const PtrBatchW &ev, const PtrBatchW &od, const u64 *pk, const u64 *cj, int nq, int nb, const u64 *iu,
                int logN, cudaStream_t s) {
    if (nb > HB_PTR_BATCH) throw std::invalid_argument("lane_split: bad batch");
    const size_t n = (size_t)(2 * nq) << logN;
    unsigned g = grid1d(n, 256);
    const unsigned cap = (148u * 32u + nb - 1) / nb;
    if (g > cap) g = cap < 1 ? 1 : cap;
    ProfScope ps(KC_ELEMENTWISE, 32.0 * n * nb, (double)n * nb, s, 1);
    k_lane_split<<<dim3(g, nb), 256, 0, s>>>(ev, od, pk, cj, nq, iu, logN);
    check_launch("lane_split");
}

// bootstrapping's ModRaise: out[pl][i][n] = centred(co[pl][n] mod q_0) mod q_i
__global__ void k_mod_raise(u64 *out, const u64 *co, int nq, int logN) {
    const size_t per = (size_t)nq << logN, n = 2 * per;
    const u64 q0 = c_pc[0].q;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
        const int pl = (int)(idx / per);
        const size_t rem = idx - (size_t)pl * per;
        const int i = (int)(rem >> logN);
        const u64 v = co[((size_t)pl << logN) + (rem & ((1u << logN) - 1))];
        const PrimeConst &pc = c_pc[i];
        if (v <= q0 / 2) {
            out[idx] = mul_shoup(v, 1ull, pc.onep, pc.q);
        } else {
            const u64 m = mul_shoup(q0 - v, 1ull, pc.onep, pc.q);
            out[idx] = m ? pc.q - m : 0;
        }
    }
}
void mod_raise_rows(u64 *out, const u64 *co, int nq, int logN, cudaStream_t s) {
    const size_t n = ((size_t)2 * nq) << logN;
    unsigned g = grid1d(n, 256);
    if (g > 148u * 64u) g = 148u * 64u;
    ProfScope ps(KC_ELEMENTWISE, 8.0 * n + 16.0 * (1 << logN), (double)n, s, 1);
    k_mod_raise<<<g, 256, 0, s>>>(out, co, nq, logN);
    check_launch("mod_raise");
}

void copy_rows(u64 *dst, const u64 *src, size_t nwords, cudaStream_t s) {
    cudaError_t e = cudaMemcpyAsync(dst, src, nwords * sizeof(u64), cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) throw std::runtime_error(std::string("copy: ") + cudaGetErrorString(e));
}

}  // namespace hb
