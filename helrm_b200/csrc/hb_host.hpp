// hb_host.hpp -- host-side number theory and the canonical-embedding
// encoder of the B200 CKKS backend.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace hb {

typedef unsigned long long u64;
typedef unsigned __int128 hu128;
typedef __int128 hi128;

inline u64 h_mulm(u64 a, u64 b, u64 q) { return (u64)(((hu128)a * b) % q); }
inline u64 h_addm(u64 a, u64 b, u64 q) { u64 s = a + b; return s >= q ? s - q : s; }
inline u64 h_subm(u64 a, u64 b, u64 q) { return a >= b ? a - b : a + (q - b); }
u64 h_powm(u64 b, u64 e, u64 q);
u64 h_invm(u64 a, u64 q);
inline u64 h_shoup(u64 w, u64 q) { return (u64)(((hu128)w << 64) / q); }
unsigned h_brv(unsigned x, int bits);

bool is_prime_u64(u64 n);

// One NTT-friendly prime per bit size (p = 1 mod 2N), nearest to 2^bits
// with the candidate below tried first at each distance, distinct from
// every prime already in `used` (which grows).  Same rule as the
// reference's Cheddar wrapper, orion/backend/cheddar/bindings.py:108-132.
std::vector<u64> gen_primes(const std::vector<int> &bits, int logn, std::vector<u64> &used);

// psi = x^((q-1)/2N) for the smallest x >= 2 giving a primitive 2N-th root.
u64 find_psi(u64 q, int logn);

// Garner's mixed-radix constants over primes[0..n) (the device decoder's
// centred CRT; encoding and decoding both run on the device).
struct CrtPlan {
    int n = 0;
    std::vector<u64> primes;
    std::vector<u64> minv;        // (prod_{k<i} q_k)^-1 mod q_i
    std::vector<u64> mmod;        // [i*n + k] = prod_{j<k} q_j mod q_i
    explicit CrtPlan(const u64 *p, int count);
};

}  // namespace hb
