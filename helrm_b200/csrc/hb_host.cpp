// hb_host.cpp -- host-side number theory and canonical-embedding encoder.
#include "hb_host.hpp"

#include <cmath>
#include <stdexcept>

namespace hb {

u64 h_powm(u64 b, u64 e, u64 q) {
    u64 r = 1 % q;
    b %= q;
    while (e) {
        if (e & 1) r = h_mulm(r, b, q);
        b = h_mulm(b, b, q);
        e >>= 1;
    }
    return r;
}

u64 h_invm(u64 a, u64 q) { return h_powm(a % q, q - 2, q); }

unsigned h_brv(unsigned x, int bits) {
    unsigned r = 0;
    for (int i = 0; i < bits; i++) {
        r = (r << 1) | (x & 1);
        x >>= 1;
    }
    return r;
}

// Deterministic Miller-Rabin, exact for 64-bit inputs with the first
// twelve primes as witnesses (the witness set the reference uses,
// orion/backend/cheddar/bindings.py:77).
bool is_prime_u64(u64 n) {
    static const u64 W[12] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
    if (n < 2) return false;
    for (u64 p : W)
        if (n % p == 0) return n == p;
    u64 d = n - 1;
    int r = 0;
    while ((d & 1) == 0) {
        d >>= 1;
        r++;
    }
    for (u64 a : W) {
        u64 x = h_powm(a, d, n);
        if (x == 1 || x == n - 1) continue;
        bool comp = true;
        for (int i = 0; i < r - 1; i++) {
            x = h_mulm(x, x, n);
            if (x == n - 1) {
                comp = false;
                break;
            }
        }
        if (comp) return false;
    }
    return true;
}

std::vector<u64> gen_primes(const std::vector<int> &bits, int logn, std::vector<u64> &used) {
    const hi128 m = (hi128)1 << (logn + 1);
    std::vector<u64> out;
    for (int b : bits) {
        if (!(b > 2 && b < 63)) throw std::invalid_argument("prime bit size out of range for uint64");
        const hi128 target = (hi128)1 << b;
        u64 found = 0;
        for (hi128 k = 1; !found; k++) {
            const hi128 cands[2] = {target + 1 - k * m, target + 1 + k * m};
            for (hi128 cd : cands) {
                if (cd < 3 || cd >= ((hi128)1 << 63)) continue;
                u64 c = (u64)cd;
                bool dup = false;
                for (u64 u : used)
                    if (u == c) {
                        dup = true;
                        break;
                    }
                if (dup) continue;
                if (is_prime_u64(c)) {
                    found = c;
                    break;
                }
            }
        }
        used.push_back(found);
        out.push_back(found);
    }
    return out;
}

u64 find_psi(u64 q, int logn) {
    const u64 N = 1ull << logn;
    for (u64 x = 2;; x++) {
        u64 g = h_powm(x, (q - 1) / (2 * N), q);
        if (h_powm(g, N, q) == q - 1) return g;
    }
}

namespace {

struct cld {
    long double re, im;
};

// In-place radix-2 DFT: forward computes sum_n a[n] w^{+rn}, inverse the
// w^{-rn} sum (no normalisation), w = exp(2 pi i / n).
void fft_ld(std::vector<cld> &a, int logn, bool inverse) {
    const int n = 1 << logn;
    for (int i = 0; i < n; i++) {
        int j = (int)h_brv((unsigned)i, logn);
        if (j > i) std::swap(a[i], a[j]);
    }
    const long double PI = 3.141592653589793238462643383279502884L;
    std::vector<cld> w(n / 2);
    for (int k = 0; k < n / 2; k++) {
        long double ang = 2.0L * PI * k / n * (inverse ? -1.0L : 1.0L);
        w[k] = {cosl(ang), sinl(ang)};
    }
    for (int len = 2; len <= n; len <<= 1) {
        const int half = len >> 1, step = n / len;
        for (int s = 0; s < n; s += len)
            for (int k = 0; k < half; k++) {
                const cld wk = w[k * step];
                const cld u = a[s + k], v = a[s + k + half];
                const cld tv = {v.re * wk.re - v.im * wk.im, v.re * wk.im + v.im * wk.re};
                a[s + k] = {u.re + tv.re, u.im + tv.im};
                a[s + k + half] = {u.re - tv.re, u.im - tv.im};
            }
    }
}

}  // namespace

void decode_coeffs(int logn, const std::vector<long double> &coeffs, long double scale,
                   double *vals_out) {
    const int N = 1 << logn, S = N / 2;
    const u64 twoN = 2ull * N;
    const long double PI = 3.141592653589793238462643383279502884L;
    std::vector<cld> w(N);
    for (int n = 0; n < N; n++) {
        long double ang = PI * n / N;
        w[n] = {coeffs[n] * cosl(ang), coeffs[n] * sinl(ang)};
    }
    fft_ld(w, logn, false);
    u64 e = 1;
    for (int j = 0; j < S; j++) {
        vals_out[2 * j] = (double)(w[(e - 1) / 2].re / scale);
        vals_out[2 * j + 1] = (double)(w[(e - 1) / 2].im / scale);
        e = (e * 5) % twoN;
    }
}

CrtPlan::CrtPlan(const u64 *p, int count) : n(count), primes(p, p + count) {
    minv.resize(n);
    mmod.assign((size_t)n * n, 0);
    mld.resize(n);
    long double M = 1.0L;
    for (int k = 0; k < n; k++) {
        mld[k] = M;
        M *= (long double)primes[k];
    }
    for (int i = 0; i < n; i++) {
        const u64 q = primes[i];
        u64 m = 1 % q;
        for (int k = 0; k < n; k++) {
            mmod[(size_t)i * n + k] = m;
            m = h_mulm(m, primes[k] % q, q);
        }
        minv[i] = h_invm(mmod[(size_t)i * n + i], q);
    }
}

long double crt_centered(const u64 *res, const CrtPlan &P) {
    const int n = P.n;
    u64 d[64], r[64];
    bool neg = false;
    for (int pass = 0; pass < 2; pass++) {
        for (int i = 0; i < n; i++) r[i] = pass ? (res[i] ? P.primes[i] - res[i] : 0) : res[i];
        for (int i = 0; i < n; i++) {
            const u64 q = P.primes[i];
            u64 acc = 0;
            for (int k = 0; k < i; k++) acc = h_addm(acc, h_mulm(d[k] % q, P.mmod[(size_t)i * n + k], q), q);
            d[i] = h_mulm(h_subm(r[i] % q, acc, q), P.minv[i], q);
        }
        if (pass == 1) break;
        // V > (Q-1)/2 iff its mixed-radix digits exceed (q_k-1)/2 read from the top
        bool gt = false;
        for (int i = n - 1; i >= 0; i--) {
            u64 h = (P.primes[i] - 1) / 2;
            if (d[i] > h) { gt = true; break; }
            if (d[i] < h) { gt = false; break; }
        }
        if (!gt) break;
        neg = true;
    }
    long double v = 0.0L;
    for (int i = 0; i < n; i++) v += (long double)d[i] * P.mld[i];
    return neg ? -v : v;
}

}  // namespace hb
