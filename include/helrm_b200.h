/*
 * helrm_b200.h -- C ABI of the B200-native CKKS backend for HE-LRM.
 *
 * Drop-in boundary for the reference's pluggable CKKS backend.  The
 * reference binds two backends behind the same integer-handle surface:
 * a Go c-shared library through ctypes (Lattigo,
 * orion/backend/lattigo/bindings.py:9-815) and a pybind11 module (Cheddar,
 * orion/backend/cheddar/ext/cheddar_pybind.cu:2403-2551).  Every entry
 * point below replaces one function of that surface; the comment names
 * the reference declaration it stands for.
 *
 * Conventions (all entry points):
 *   - return 0 on success, a negative HB_E* code on failure; the message of
 *     the last failure is available from helrm_LastError();
 *   - objects live in the library; callers hold int handles (> 0); "New"
 *     functions write the new handle through an out pointer, in-place
 *     functions reuse the handle they were given;
 *   - plain pointers and sizes only; arrays are caller-allocated;
 *   - single-threaded and stateful like the reference (one scheme per
 *     process, orion/backend/lattigo/scheme.go:32); all GPU work is
 *     enqueued on the library's own stream (the asynchronous batch
 *     transfers on two more, ordered with events) and synchronised only
 *     where a result crosses to the host.
 * Levels follow Orion: a ciphertext at level l has l+1 residue limbs, a
 * fresh one sits at len(LogQ)-1 (orion/backend/python/parameters.py:258).
 * Rotation by k is a left shift, rot(ct,k)[i] = ct[i+k], shifts reduced to
 * [0, slots) (cheddar_pybind.cu:1858-1870; tests/oracle/assumptions.md:5-9).
 */
#ifndef HELRM_B200_H
#define HELRM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HB_OK 0
#define HB_EINVAL -1    /* bad argument (Python: ValueError) */
#define HB_ENOENT -2    /* unknown handle (Python: IndexError / KeyError) */
#define HB_ESTATE -3    /* scheme not set up, level/scale precondition (RuntimeError) */
#define HB_ECUDA -4     /* CUDA error (RuntimeError) */
#define HB_ENOMEM -5    /* device allocation failed (MemoryError) */
#define HB_ENOTSUP -6   /* not implemented (NotImplementedError) */

/* Message of the most recent failure ("" if none). */
const char *helrm_LastError(void);

/* ---- lifecycle ---------------------------------------------------------- */

/* NewScheme -- orion/backend/lattigo/scheme.go:35-86 (bound at
 * lattigo/bindings.py:149-187); Cheddar setup_scheme cheddar_pybind.cu:359-468.
 * Primes are generated like the reference's Cheddar wrapper
 * (orion/backend/cheddar/bindings.py:108-132).  dnum <= 0 selects Lattigo's
 * default (digits of len(logp) primes).  seed fixes the keys' and
 * encryptions' counter-based sampler.  device is the CUDA ordinal. */
int helrm_NewScheme(int logn, const int *logq, int nlogq, const int *logp, int nlogp, int logscale,
                    int hamming_weight, int dnum, uint64_t seed, int device);
/* DeleteScheme -- scheme.go:89; cheddar delete_scheme. */
int helrm_DeleteScheme(void);
/* GetModuliChain / GetAuxModuliChain -- tensors.go:105-130; cheddar bindings.py:1262-1276. */
int helrm_GetModuliChain(uint64_t *out, int cap, int *n);
int helrm_GetAuxModuliChain(uint64_t *out, int cap, int *n);
/* slots (N/2), max level, log2 N, alpha, dnum -- parameters.py:237-264 */
int helrm_GetSchemeInfo(int *logn, int *slots, int *max_level, int *alpha, int *dnum);
/* Host-only: the prime rule NewScheme uses (orion/backend/cheddar/bindings.py:108-132).
 * Writes n primes for the bit sizes in bits; `used` (nused entries) are
 * excluded.  Needs no GPU and no scheme. */
int helrm_GenPrimes(int logn, const int *bits, int n, const uint64_t *used, int nused, uint64_t *out);

/* ---- keys ---------------------------------------------------------------- */
/* keygenerator.go:18-36; cheddar bindings.py:458-473 */
int helrm_GenerateSecretKey(void);
int helrm_GeneratePublicKey(void);
int helrm_GenerateRelinearizationKey(void);
/* conjugation key (GenerateEvaluationKeys, keygenerator.go:33; evaluator.go:55-66) */
int helrm_GenerateEvaluationKeys(void);
/* AddRotationKey -- evaluator.go:38-53; cheddar_pybind.cu:1872-1883 */
int helrm_AddRotationKey(int k);

/* ---- encode / decode ------------------------------------------------------- */
/* Encode -- encoder.go:16-31 (bindings.py:338-356); cheddar_pybind.cu:538-558.
 * n <= slots real values, zero padded. */
int helrm_Encode(const double *values, int n, int level, double scale, int *out_pt);
/* EncodeComplex -- interleaved (re, im) pairs, n pairs. cheddar_pybind.cu:563-578 */
int helrm_EncodeComplex(const double *interleaved, int n, int level, double scale, int *out_pt);
/* Decode / DecodeComplex -- encoder.go:33-48,76-91; cheddar_pybind.cu:580-603.
 * Writes min(cap, slots) values (pairs for complex) and the count to *n. */
int helrm_Decode(int pt, double *out, int cap, int *n);
int helrm_DecodeComplex(int pt, double *out, int cap, int *n);

/* ---- encrypt / decrypt ------------------------------------------------------ */
/* Encrypt / Decrypt -- encryptor.go:20-38; cheddar_pybind.cu:621-627,680-696 */
int helrm_Encrypt(int pt, int *out_ct);
int helrm_Decrypt(int ct, int *out_pt);
/* EncryptSeeded / DropAx / ExpandSeededAx -- cheddar_pybind.cu:638-660 */
int helrm_EncryptSeeded(int pt, uint64_t seed, int *out_ct);
int helrm_DropAx(int ct);
int helrm_ExpandSeededAx(int ct, uint64_t seed);

/* ---- ciphertext arithmetic (evaluator.go:69-364; cheddar_pybind.cu:702-1856) -- */
int helrm_AddCiphertextNew(int a, int b, int *out);
int helrm_AddCiphertext(int a, int b);
int helrm_SubCiphertextNew(int a, int b, int *out);
int helrm_SubCiphertext(int a, int b);
int helrm_MulRelinCiphertextNew(int a, int b, int *out);
int helrm_MulRelinCiphertext(int a, int b);
/* Negate -- a new ciphertext -ct (evaluator.go:68-78, cheddar_pybind.cu:1798-1803) */
int helrm_Negate(int ct, int *out);
int helrm_AddPlaintextNew(int ct, int pt, int *out);
int helrm_AddPlaintext(int ct, int pt);
int helrm_SubPlaintextNew(int ct, int pt, int *out);
int helrm_SubPlaintext(int ct, int pt);
/* MulPlaintext[New] -- no rescale (evaluator.py:59-65 rescales) */
int helrm_MulPlaintextNew(int ct, int pt, int *out);
int helrm_MulPlaintext(int ct, int pt);
/* MulPlaintextAccumNew -- fused sum_i ct_i*pt_i, cheddar_pybind.cu:834-900 */
int helrm_MulPlaintextAccumNew(const int *cts, const int *pts, int n, int *out);
int helrm_AddScalarNew(int ct, double s, int *out);
int helrm_AddScalar(int ct, double s);
int helrm_SubScalarNew(int ct, double s, int *out);
int helrm_SubScalar(int ct, double s);
/* MulScalarInt keeps the level; MulScalarFloat squares the scale (cheddar_pybind.cu:1722-1792) */
int helrm_MulScalarIntNew(int ct, int64_t s, int *out);
int helrm_MulScalarInt(int ct, int64_t s);
int helrm_MulScalarFloatNew(int ct, double s, int *out);
int helrm_MulScalarFloat(int ct, double s);
/* Rescale[New] -- cheddar_pybind.cu:1843-1856 */
int helrm_RescaleNew(int ct, int *out);
int helrm_Rescale(int ct);
/* AlignToLevelNew -- cheddar_pybind.cu:329-342 (drops limbs) */
int helrm_AlignToLevelNew(int ct, int level, int *out);
/* Rotate[New] -- evaluator.go:81-102; cheddar_pybind.cu:1885-1900 */
int helrm_RotateNew(int ct, int k, int *out);
int helrm_Rotate(int ct, int k);
/* RotateBatchNew -- one hoisted ModUp shared by all shifts, cheddar_pybind.cu:1986-2031 */
int helrm_RotateBatchNew(int ct, const int *ks, int n, int *outs);
/* Conjugate[New] -- evaluator.go:104-129; cheddar_pybind.cu:1812-1830 */
int helrm_ConjugateNew(int ct, int *out);
int helrm_Conjugate(int ct);

/* ---- linear transforms (lineartransform.go:37-211; cheddar bindings.py:833-1066) -- */
/* GenerateLinearTransform: n diagonals, each `width` values, row-major in
 * `data`; bsgs_ratio <= 0 means "none" (one giant group).  The diagonals are
 * encoded at the level's prime (lineartransform.go:65), so the rescaled
 * output keeps the input's scale. */
int helrm_GenerateLinearTransform(const int *diag_idxs, int n, const double *data, int width, int level,
                                  double bsgs_ratio, int *out_lt);
int helrm_EvaluateLinearTransform(int lt, int ct, int *out);
/* B200 addition: the same transform over n ciphertexts in one pass, so
 * the plaintext diagonals and evaluation keys stream once per batch. */
int helrm_EvaluateLinearTransformBatch(int lt, const int *cts, int n, int *outs);
int helrm_DeleteLinearTransform(int lt);
int helrm_GetLinearTransformRotationKeys(int lt, int *out, int cap, int *n);
/* baby-step stride chosen for the transform (bindings.py:857-862) */
int helrm_GetLinearTransformInfo(int lt, int *bs, int *ndiag, int *ngiant, int *level);
/* Hybrid-method output fold -- orion/nn/linear.py:115-117: for i in
 * 1..rotations: ct += rot(ct, slots / 2^i), applied in place to n cts. */
int helrm_HybridFoldBatch(const int *cts, int n, int rotations);
/* Rescale n ciphertexts in place. */
int helrm_RescaleBatch(const int *cts, int n);
/* out[i] = MulRelinCiphertextNew(a[i], b[i]) for n pairs, the pairs of one
 * level computed together (batch form of the per-pair call above; the
 * reference's evaluators multiply one pair per call). */
int helrm_MulRelinCiphertextBatchNew(const int *a, const int *b, int n, int *out);

/* ---- broadcast constants and the one-pass table products of the IVE lookup
 * (cheddar bindings.py:621-706; cheddar_pybind.cu:1044-1569).  A constant is
 * round(scalar * scale) mod q_i, one word per prime; a table is rows x cols
 * constants or plaintexts, row-major.  The products read every input
 * ciphertext once for all rows; outputs carry scale ct * table and are not
 * rescaled.  Ciphertexts above the table's level are read at its level;
 * primes below 2^40. */
/* EncodeConstantNew -- bindings.py:621-630 */
int helrm_EncodeConstantNew(double scalar, int level, double scale, int *out);
int helrm_DeleteConstant(int id);
/* MulConstantAccumNew -- sum_i c_i * ct_i, bindings.py:635-643 */
int helrm_MulConstantAccumNew(const int *cts, const int *consts, int n, int *out);
/* PackConstantTableNew / PackPlaintextTableNew -- bindings.py:645-686
 * (a plaintext table refers to its plaintexts by id: keep them alive) */
int helrm_PackConstantTableNew(const int *consts, int n, int rows, int *out_table);
int helrm_PackPlaintextTableNew(const int *pts, int n, int rows, int *out_table);
/* DeleteConstantTable / DeletePlaintextTable -- bindings.py:656-687 */
int helrm_DeleteTable(int table);
int helrm_GetTableShape(int table, int *rows, int *cols, int *level);
/* MulConstantMatMulNew / MulPlaintextMatMulNew -- bindings.py:659-697:
 * n = cols input ciphertexts, rows ids written to outs */
int helrm_MulTableMatMulNew(const int *cts, int n, int table, int *outs);

/* ---- upload path (cheddar_pybind.cu:538-560 Encode, 1825-1837
 * MulImaginaryUnit; orion/core/lane_packing.py:84-115) -------------------------
 * Encoding runs on the device: the slot values cross to HBM as doubles and
 * the special FFT, rounding, residues and NTT happen there.
 * EncodeBatch: count real vectors of n values each ([count][n], row-major),
 * one plaintext per vector, ids written to outs. */
int helrm_EncodeBatch(const double *values, int count, int n, int level, double scale, int *outs);
/* slot-wise multiplication by sqrt(-1): key-free, no level consumed */
int helrm_MulImaginaryUnitNew(int ct, int *out);
int helrm_MulImaginaryUnit(int ct);
/* complex-lane unpacking of n packed uploads p = (x + i y) / 2: outs[2m] = x,
 * outs[2m+1] = y of packed[m] (x = p + conj p, y = -i (p - conj p)), the
 * first num_real of them (0 <= num_real <= 2n) written to outs */
int helrm_UnpackLanes(const int *packed, int n, int num_real, int *outs);

/* ---- bootstrapping pieces (NewBootstrapper / Bootstrap, cheddar bindings.py:
 * 1326-1342 -> cheddar_pybind.cu:2049-2187; the circuit runs in the Python
 * layer over these and the operators above) ----------------------------------
 * ModRaise: a level-0 ciphertext lifted (centred) to every main prime; it
 * decrypts to m + q_0 I with I the small overflow polynomial. */
int helrm_ModRaiseNew(int ct, int *out);
/* GenerateLinearTransform with complex diagonals (cplx != 0: interleaved re,
 * im pairs, width pairs per diagonal) encoded at plaintext scale `scale`
 * (<= 0: the default scale); the transform's output scale is the input's
 * times `scale` */
int helrm_GenerateLinearTransformEx(const int *diag_idxs, int n, const double *data, int width, int level,
                                    double bsgs_ratio, int cplx, double scale, int *out_lt);

/* ---- polynomial evaluation (poly_evaluator.py:25-35; cheddar bindings.py:
 * 1102-1116 -> EvaluatePolynomialNative, cheddar_pybind.cu:2207-2262) --------
 * coeffs[0..n) ascending, n >= 3 (degree >= 2; the Python layer keeps Horner
 * below that, bindings.py:1104-1116), chebyshev != 0: sum c_j T_j(x), else
 * sum c_j x^j.  The output sits ceil(log2(n)) levels below the input
 * (orion/nn/activation.py:22-28,101-110) at exactly `scale`; the input must be
 * relinearized and hold that many levels. */
int helrm_EvaluatePolynomial(int ct, const double *coeffs, int n, int chebyshev, double scale, int *out);
/* the same polynomial over nb ciphertexts (the ids of a CipherTensor,
 * poly_evaluator.py:29-31) in batched kernels; nb ids written to outs */
int helrm_EvaluatePolynomialBatch(const int *cts, int nb, const double *coeffs, int n, int chebyshev,
                                  double scale, int *outs);
/* the evaluation plan for an input of nq rows at in_scale: info[0] levels
 * consumed, info[1] ciphertext products, info[2] rescales, info[3] baby steps */
int helrm_PolynomialPlanInfo(int nq, double in_scale, const double *coeffs, int n, int chebyshev, double scale,
                             int *info);

/* ---- metadata (tensors.go:35-104; cheddar bindings.py:1278-1320) ------------- */
int helrm_DeleteCiphertext(int ct);
int helrm_DeletePlaintext(int pt);
int helrm_GetCiphertextLevel(int ct, int *level);
int helrm_GetPlaintextLevel(int pt, int *level);
int helrm_GetCiphertextScale(int ct, double *scale);
int helrm_GetPlaintextScale(int pt, double *scale);
int helrm_SetCiphertextScale(int ct, double scale);
int helrm_SetPlaintextScale(int pt, double scale);
int helrm_GetCiphertextSlots(int ct, int *slots);
int helrm_GetPlaintextSlots(int pt, int *slots);
int helrm_SetCiphertextSlots(int ct, int slots);
int helrm_GetCiphertextDegree(int ct, int *degree);
int helrm_GetLiveCounts(int *ciphertexts, int *plaintexts);
int helrm_GetCiphertextBytes(int ct, double *bytes);
int helrm_GetMemoryMB(double *live, double *peak_live, double *keys);

/* ---- raw residues (test and wire I/O; host buffers, limb-major) ------------- */
/* words = npoly * (level+1) * N */
int helrm_GetCiphertextData(int ct, uint64_t *out, size_t words);
int helrm_NewCiphertextFromData(const uint64_t *data, int level, int npoly, double scale, int *out);
/* plaintext rows: (level+1) q rows, plus K special-prime rows when ext */
int helrm_GetPlaintextData(int pt, uint64_t *out, size_t words);
int helrm_NewPlaintextFromData(const uint64_t *data, int level, int ext, double scale, int *out);
/* evaluation keys [dnum][2][L+K][N]; galois 0 selects the relinearisation key */
int helrm_GetKeyData(uint64_t galois, uint64_t *out, size_t words);
/* secret key, NTT form over all L+K primes [L+K][N] (tests only) */
int helrm_GetSecretKeyData(uint64_t *out, size_t words);
/* extended-basis plaintext of diagonal `k` of a transform */
int helrm_GetLinearTransformPlaintext(int lt, int k, uint64_t *out, size_t words);

/* ---- asynchronous batch transfers (no reference counterpart: the reference
 * uploads with Encrypt on the device and reads results through Decrypt/Decode,
 * examples/criteo/bench_sweep.py:225-243).  Copies run on two more streams,
 * one per direction, and overlap the arithmetic; the library orders them with
 * events.  Host buffers should be pinned (page-locked) for the copies to be
 * asynchronous, and must stay valid and unmodified until helrm_TransferSync
 * returns. ------------------------------------------------------------------- */
/* n ciphertexts [npoly][level+1][N] from host[i]; ids written to out_ids.
 * Work issued later on the ciphertexts waits for the copies on the device. */
int helrm_UploadCiphertextsAsync(const uint64_t *const *host, int n, int level, int npoly, double scale,
                                 int *out_ids);
/* copy n ciphertexts to host[i] (each at least words_each words) after all
 * work issued so far; deleting them afterwards is safe (the memory is freed
 * behind the copy). */
int helrm_DownloadCiphertextsAsync(const int *ids, int n, uint64_t *const *host, size_t words_each);
/* wait for every asynchronous transfer */
int helrm_TransferSync(void);

/* ---- device-buffer exchange of ciphertexts between ranks (no reference
 * counterpart: the reference runs on one GPU; this is the table-sharded
 * layer's exchange step).  The buffers are device memory of the scheme's
 * GPU, e.g. the tensor a collective reduces. ------------------------------ */
/* copy n ciphertexts' residues [npoly][level+1][N] into d_out, item i at
 * i * words_each; returns after the copies have finished */
int helrm_CiphertextsToDevice(const int *ids, int n, uint64_t *d_out, size_t words_each);
/* n new ciphertexts [npoly][level+1][N] from d_in holding per-limb 64-bit
 * sums of residues (several ranks' partial ciphertexts added as integers);
 * every word is reduced modulo its limb's prime on import.  d_in must be
 * complete before the call (the library orders only its own stream). */
int helrm_NewCiphertextsFromDeviceSum(const uint64_t *d_in, int n, int level, int npoly, double scale,
                                      int *out_ids);

/* ---- kernel-level entry points on device pointers (microbenchmarks) --------- */
/* Forward / inverse NTT in place on nrows limbs laid out as blocks of
 * `per` rows (nq main-prime rows then special-prime rows). */
int helrm_kernel_ntt(uint64_t *d_data, int nrows, int per, int nq, int inverse, void *stream);
/* out[r][t] = in[r][tau_g(t)] on nrows limbs */
int helrm_kernel_automorphism(const uint64_t *d_in, uint64_t *d_out, int nrows, uint64_t galois, void *stream);
/* nbatch ciphertexts [2][nq] -> [2][nq-1], rounded rescale by q_{nq-1} */
int helrm_kernel_rescale(const uint64_t *d_in, uint64_t *d_out, int nq, int nbatch, void *stream);
/* out[2][nq] = sum_t ct_t[2][nq] * pt_t[nq] over nterms (device pointer arrays in host memory) */
int helrm_kernel_mac(const uint64_t *const *d_cts, const uint64_t *const *d_pts, int nterms, int nq,
                     uint64_t *d_out, void *stream);
/* Hoisted rotations of nbatch ciphertexts (level nq-1) by nrot Galois
 * elements sharing one ModUp per ciphertext.  Keys must exist
 * (helrm_AddRotationKey).  d_out: [nrot][nbatch][2][nq][N]. */
int helrm_kernel_rotate_hoisted(const uint64_t *d_in, int nq, int nbatch, const int *ks, int nrot,
                                uint64_t *d_out, void *stream);
/* Same result as helrm_kernel_rescale, but the call allocates no device
 * memory.  No counterpart in the reference, whose Python operators allocate
 * freely.  Its temporaries (the INTT of the last limb and the correction
 * term, nbatch*2*nq*N words in all) come from one fixed array compiled into
 * the library, HELRM_RESCALE_SCRATCH_WORDS words (32 MiB) per device: one
 * ciphertext of N = 2^16 at 24 limbs fits.  Larger requests fail with
 * HB_EINVAL before any work is issued.  helrm_NewScheme looks up that
 * array's device address once, with the scheme's device current, so the
 * call itself does no set-up.  All calls on a device share the array: calls
 * whose GPU work overlaps (unordered streams, several host threads) race and
 * corrupt each other's output. */
#define HELRM_RESCALE_SCRATCH_WORDS (4u << 20)
int helrm_kernel_rescale_noalloc(const uint64_t *d_in, uint64_t *d_out, int nq, int nbatch, void *stream);
/* synchronise the library stream */
int helrm_Synchronize(void);

/* ---- measurement (no reference counterpart; the reference times with
 * torch.cuda.synchronize + wall clock, examples/criteo/bench_sweep.py:192-222) -- */
/* CUDA events on the library stream around a region of work. */
int helrm_TimerStart(void);
int helrm_TimerStop(double *ms);
/* Per-kernel-class CUDA-event timing on the launching stream, with each
 * launch's algorithmic bytes and modular products (NTT: butterflies).
 * Enabling resets the statistics. */
int helrm_ProfileEnable(int on);
int helrm_ProfileRead(double *ms, double *bytes, double *work, uint64_t *launches, int cap, int *nclasses);
int helrm_KernelClassName(int cls, char *out, int cap);
/* cudaProfilerStart / cudaProfilerStop around a region (for an external
 * profiler started with profiling off) */
int helrm_ProfilerRange(int on);
/* number of kernels this library has launched since it was loaded */
int helrm_GetLaunchCount(uint64_t *n);
/* number of device-pool allocations the current scheme has made */
int helrm_GetAllocCount(uint64_t *n);

#ifdef __cplusplus
}
#endif
#endif /* HELRM_B200_H */
