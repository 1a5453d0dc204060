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

CrtPlan::CrtPlan(const u64 *p, int count) : n(count), primes(p, p + count) {
    minv.resize(n);
    mmod.assign((size_t)n * n, 0);
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

}  // namespace hb
