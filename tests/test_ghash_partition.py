"""CPU model of the seal / open-GHASH kernels' partition of GHASH, checked
against the oracle's serial GHASH (oracle_ghash_ct).

The kernels split the n ciphertext blocks over G CTAs of J rows x T threads
(CTA c covers [n - (G-c)JT, n - (G-1-c)JT), leading slots below block 0
skipped). Each thread runs R Horner chains (chain k takes its rows r = k mod R,
multiplier H^(R*T)), combines them with H^T into sum_r X_r H^(T(J-1-r)), the T
thread shares are folded with H^(2^l), and each CTA's fold is scaled by
H^(d_c), d_c = (G-1-c)JT + 2; the length block contributes L*H. R = 1 in
seal_kernel, 2 in open_ghash_kernel. This model mirrors horner_grid() in
confkv_b200/csrc/gpu_aesgcm.cu and the algebra of chain_push_dyn /
chains_combine / fold_partials / cta_accumulate in kernels.cuh.
"""

import numpy as np
import pytest

T = 512
FOLD_LEVELS = 9
ONE = b"\x80" + bytes(15)


def xor(a: bytes, b: bytes) -> bytes:
    return (int.from_bytes(a, "big") ^ int.from_bytes(b, "big")).to_bytes(16, "big")


def horner_grid(n: int, num_sms: int) -> tuple[int, int]:
    per_wave = num_sms * T
    j = max(1, -(-n // per_wave))
    span = j * T
    return j, -(-n // span)


def model_ghash(oracle, h: bytes, ct: bytes, num_sms: int, chains: int) -> bytes:
    mul = oracle.gf_mul

    def power(e: int) -> bytes:
        r, b = ONE, h
        while e:
            if e & 1:
                r = mul(r, b)
            b = mul(b, b)
            e >>= 1
        return r

    P = len(ct)
    n = -(-P // 16)
    padded = ct + bytes(16 * n - P)
    blocks = [padded[16 * i:16 * i + 16] for i in range(n)]
    iters, grid = horner_grid(n, num_sms)
    span = iters * T
    ht = power(T)
    hrt = power(chains * T)
    fold_pows = [power(1 << l) for l in range(FOLD_LEVELS)]
    acc = bytes(16)
    for c in range(grid):
        base = n - (grid - c) * span
        q = [[bytes(16)] * chains for _ in range(T)]
        for r in range(iters):
            for t in range(T):
                i = base + r * T + t
                x = blocks[i] if i >= 0 else bytes(16)
                q[t][r % chains] = xor(mul(q[t][r % chains], hrt), x)
        part = []
        for t in range(T):
            share = bytes(16)
            for d in range(chains - 1, -1, -1):
                k = (iters - 1 - d) % chains
                share = q[t][k] if d == chains - 1 else xor(mul(share, ht), q[t][k])
            part.append(share)
        for l in range(FOLD_LEVELS):
            for p in range(T >> (l + 1)):
                left = p << (l + 1)
                part[left] = xor(mul(part[left], fold_pows[l]), part[left + (1 << l)])
        d = (grid - 1 - c) * span + 2
        acc = xor(acc, mul(part[0], power(d)))
    lenblk = bytes(8) + (8 * P).to_bytes(8, "big")
    return xor(acc, mul(lenblk, h))


@pytest.mark.parametrize("chains", [1, 2, 3, 4])
@pytest.mark.parametrize("size,num_sms", [(1, 148), (16, 148), (17, 4), (4096, 148), (16 * 700 + 5, 2),
                                          (16 * 1024, 4), (16 * 1537 + 9, 3), (16 * 3000, 2)])
def test_partitioned_ghash_matches_serial(oracle, size, num_sms, chains):
    rng = np.random.default_rng(size * 7 + num_sms)
    h = rng.bytes(16)
    ct = rng.bytes(size)
    assert model_ghash(oracle, h, ct, num_sms, chains) == oracle.ghash_ct(h, ct)


def test_grid_covers_blocks_once():
    for n in (1, 255, 256, 257, 37888, 37889, 131072, 2097152, 655360, 67108864):
        iters, grid = horner_grid(n, 148)
        span = iters * T
        assert grid <= 148
        assert grid * span >= n
        # only CTA 0 may start below block 0, and by less than one CTA span
        assert n - grid * span > -span
