"""CPU model of the streaming record decode's CRC-32 arithmetic (csrc/records.cu,
record_stream_kernel and record_stream_plan), checked against zlib: lanes fold 16-byte pieces
into per-lane registers over "piece, 496 zero bytes" streams with nibble tables, the registers
are moved to the row end with per-lane constants, runs of whole rows get a per-chunk constant
(negative powers of x included), and zlib's preset is added at the end. Small payloads and a
few row/chunk splits, so it runs in seconds; the kernel itself is tested on the GPU."""

from __future__ import annotations

import random
import zlib

import pytest

POLY = 0xEDB88320
ONE = 1 << 31  # x^0 in the reflected representation


def mulx(a: int) -> int:
    return (a >> 1) ^ (POLY if a & 1 else 0)


def divx(c: int) -> int:  # undoes one multiplication by x
    b = c >> 31
    t = c ^ (POLY if b else 0)
    return ((t << 1) & 0xFFFFFFFF) | b


def mulmod(a: int, b: int) -> int:
    p, m = 0, 1 << 31
    while m:
        if a & m:
            p ^= b
        b = mulx(b)
        m >>= 1
    return p


def xpow(e: int) -> int:
    base = mulx(ONE) if e >= 0 else divx(ONE)
    e, acc = abs(e), ONE
    while e:
        if e & 1:
            acc = mulmod(acc, base)
        base = mulmod(base, base)
        e >>= 1
    return acc


def nibble_table(c: int, j: int) -> list[int]:
    """(n << 4 j) * c mod P for n < 16, as the kernel's nibble_table builds it."""
    for _ in range(28 - 4 * j):
        c = mulx(c)
    b3 = c
    b2 = mulx(b3)
    b1 = mulx(b2)
    b0 = mulx(b1)
    basis = [b0, b1, b2, b3]
    return [sum_xor(basis[q] for q in range(4) if n >> q & 1) for n in range(16)]


def sum_xor(vals) -> int:
    r = 0
    for v in vals:
        r ^= v
    return r


def stream_crc(record: bytes, payload_len: int, max_chunks: int, seed: int) -> int:
    end = 52 + payload_len
    q_last = (end - 1) // 16
    nrows = (q_last - 2 + 31) // 32
    rows_per_chunk = -(-nrows // max_chunks)
    nchunks = -(-nrows // rows_per_chunk)
    tz = 512 * nrows - 4 - payload_len
    word_tabs = [[nibble_table(xpow(8 * (512 - 4 * w)), j) for j in range(8)] for w in range(4)]
    lane_tabs = [[nibble_table(xpow(128 * (31 - l)), j) for j in range(8)] for l in range(32)]
    chunk_shift = [xpow(4096 * (nrows - min((c + 1) * rows_per_chunk, nrows)) - 128 * 31 - 8 * tz)
                   for c in range(nchunks)]

    def piece(q: int) -> list[int]:
        b = bytearray(record[16 * q:16 * q + 16].ljust(16, b"\0"))
        for i in range(16):  # bytes outside the payload count as zeros
            if not 52 <= 16 * q + i < end:
                b[i] = 0
        return [int.from_bytes(b[4 * w:4 * w + 4], "little") for w in range(4)]

    rnd = random.Random(seed)
    acc, c = 0, 0
    while c < nchunks:  # runs of whole chunks, as the warps' ranges cut them
        cend = min(nchunks, c + rnd.randint(1, 3))
        k0, k1 = c * rows_per_chunk, min(cend * rows_per_chunk, nrows)
        S = [0] * 32
        for k in range(k0, k1):
            for lane in range(32):
                p = piece(3 + 32 * k + lane)
                p[0] ^= S[lane]
                S[lane] = sum_xor(word_tabs[w][j][(p[w] >> 4 * j) & 15]
                                  for w in range(4) for j in range(8))
        g = sum_xor(lane_tabs[lane][j][(S[lane] >> 4 * j) & 15]
                    for lane in range(32) for j in range(8))
        acc ^= mulmod(g, chunk_shift[cend - 1])
        c = cend
    init_term = mulmod(0xFFFFFFFF, xpow(8 * payload_len))
    return (~(acc ^ init_term)) & 0xFFFFFFFF


@pytest.mark.parametrize("payload_len,max_chunks", [(16, 128), (496, 128), (512, 2),
                                                    (4096, 3), (8208, 4), (18432, 128)])
def test_stream_crc_model_equals_zlib(payload_len, max_chunks):
    rnd = random.Random(payload_len)
    payload = bytes(rnd.getrandbits(8) for _ in range(payload_len))
    stride = -(-(52 + payload_len) // 4096) * 4096
    header = bytes(rnd.getrandbits(8) for _ in range(52))   # must not enter the CRC
    padding = bytes(rnd.getrandbits(8) for _ in range(stride - 52 - payload_len))
    record = header + payload + padding
    assert stream_crc(record, payload_len, max_chunks, seed=payload_len) == zlib.crc32(payload)
