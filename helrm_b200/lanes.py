"""Complex-lane packing of client uploads on the B200 backend.

The reference packs two real ciphertext-sized chunks into the real and
imaginary lanes of one upload and splits them on the server with one
conjugation each (orion/core/lane_packing.py:42-115, used by
examples/criteo/bench_sweep.py for the HE-LRM selector upload):

    p = (x + i y) / 2,   x = p + conj(p),   y = -i (p - conj(p)).

Chunk 2m goes to the real lane and chunk 2m+1 to the imaginary lane of
packed ciphertext m, so every unpacked ciphertext covers the slot range an
unpacked upload would have, and the consuming layer is unchanged.  The
server side here is ``B200Library.UnpackLanes``: one batched conjugation
key switch for all packed ciphertexts and both lanes written in one pass,
residue for residue what the reference's op-by-op sequence (ConjugateNew,
AddCiphertextNew, SubCiphertextNew, MulImaginaryUnit, Negate) produces.
"""
from __future__ import annotations

import numpy as np


def plan_packing(num_elements: int, num_slots: int) -> tuple[int, int]:
    """(real ciphertexts, packed ciphertexts) of a num_elements upload
    (lane_packing.py:42-52)."""
    num_real = -(-int(num_elements) // int(num_slots))
    return num_real, -(-num_real // 2)


def is_profitable(num_elements: int, num_slots: int) -> bool:
    """Packing pays from two real ciphertexts on (lane_packing.py:55-57)."""
    return plan_packing(num_elements, num_slots)[0] >= 2


def pack_lanes(values, num_slots: int):
    """Client side (lane_packing.py:60-81): the flat complex vector of
    ceil(n/2) * num_slots entries holding 0.5 (chunk_2m + i chunk_2m+1),
    and n, the number of real ciphertexts the server rebuilds."""
    flat = np.asarray(values, dtype=np.float64).ravel()
    pad = (-flat.size) % num_slots
    if pad:
        flat = np.concatenate([flat, np.zeros(pad)])
    chunks = flat.reshape(-1, num_slots)
    num_real = chunks.shape[0]
    if num_real % 2:
        chunks = np.concatenate([chunks, np.zeros((1, num_slots))])
    packed = 0.5 * (chunks[0::2] + 1j * chunks[1::2])
    return packed.ravel(), num_real


def encode_packed(backend, packed, num_slots: int, level: int, scale) -> list[int]:
    """One plaintext per packed chunk (interleaved re, im through EncodeComplex)."""
    z = np.asarray(packed, dtype=np.complex128).reshape(-1, num_slots)
    ids = []
    for row in z:
        inter = np.stack([row.real, row.imag], axis=-1).ravel()
        ids.append(backend.EncodeComplex(inter, level, scale))
    return ids


def unpack_lanes(backend, packed_ids, num_real: int) -> list[int]:
    """Server side (lane_packing.py:84-115): the num_real real-lane
    ciphertexts, in order, at the packed ciphertexts' level and scale."""
    return backend.UnpackLanes(list(packed_ids), int(num_real))
