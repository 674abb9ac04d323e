"""The register-streamed small-batch GEMM's fragment mapping, checked on the CPU.

`gemm_rs_kernel` (strands_decider_b200/csrc/gemm_rs.cu) feeds mma.sync m16n8k16 with the weights
as the A operand and 8 tokens as the B operand, but it does not give the MMA's k-slots the
columns in their natural order: lane (g, t) holds columns 16 t .. 16 t + 15 of one 64-column
k-block for weight rows g and g + 8 and for token g, and MMA j of the block takes the pairs 2j
and 2j + 1 of them. This emulates the PTX fragment layouts of mma.m16n8k16 (A: a0 a1 = row g,
k 2t, 2t+1; a2 a3 = row g+8; a4 a5 = row g, k 2t+8, 2t+9; a6 a7 = row g+8; B: b0 b1 = k 2t, 2t+1,
column g; b2 b3 = k 2t+8, 2t+9; C: c0 c1 = row g, columns 2t, 2t+1; c2 c3 = row g+8) in float64
and checks that the four MMAs of a k-block, fed that way, sum to W X^T for the block.
"""

from __future__ import annotations

import numpy as np


def _mma_16816(a_regs, b_regs):
    """One warp's m16n8k16: a_regs[lane] = 4 pairs, b_regs[lane] = 2 pairs (each pair = the
    register's low and high bf16, here float64); returns c[lane] = 4 floats."""
    A = np.zeros((16, 16))
    B = np.zeros((16, 8))
    for lane in range(32):
        g, t = lane // 4, lane % 4
        (a01, a23, a45, a67) = a_regs[lane]
        A[g, 2 * t: 2 * t + 2] = a01
        A[g + 8, 2 * t: 2 * t + 2] = a23
        A[g, 2 * t + 8: 2 * t + 10] = a45
        A[g + 8, 2 * t + 8: 2 * t + 10] = a67
        (b01, b23) = b_regs[lane]
        B[2 * t: 2 * t + 2, g] = b01
        B[2 * t + 8: 2 * t + 10, g] = b23
    C = A @ B
    out = []
    for lane in range(32):
        g, t = lane // 4, lane % 4
        out.append(np.array([C[g, 2 * t], C[g, 2 * t + 1], C[g + 8, 2 * t], C[g + 8, 2 * t + 1]]))
    return out


def test_register_path_kslot_order_gives_the_product():
    rng = np.random.default_rng(0)
    W = rng.standard_normal((16, 64))   # one 16-row weight tile, one 64-column k-block
    X = rng.standard_normal((8, 64))    # one 8-token tile
    acc = [np.zeros(4) for _ in range(32)]
    for j in range(4):
        a_regs, b_regs = [], []
        for lane in range(32):
            g, t = lane // 4, lane % 4
            P = [W[g, 16 * t + 2 * p: 16 * t + 2 * p + 2] for p in range(8)]      # row g's 8 pairs
            Q = [W[g + 8, 16 * t + 2 * p: 16 * t + 2 * p + 2] for p in range(8)]  # row g + 8's
            Xp = [X[g, 16 * t + 2 * p: 16 * t + 2 * p + 2] for p in range(8)]     # token g's
            a_regs.append((P[2 * j], Q[2 * j], P[2 * j + 1], Q[2 * j + 1]))
            b_regs.append((Xp[2 * j], Xp[2 * j + 1]))
        for lane, c in enumerate(_mma_16816(a_regs, b_regs)):
            acc[lane] += c
    want = W @ X.T   # [weight row][token]
    for lane in range(32):
        g, t = lane // 4, lane % 4
        np.testing.assert_allclose(acc[lane], [want[g, 2 * t], want[g, 2 * t + 1], want[g + 8, 2 * t],
                                               want[g + 8, 2 * t + 1]], rtol=1e-12, atol=1e-12)


def test_natural_order_would_differ():
    """The mapping is not vacuous: feeding the same registers as if the k-slots held the columns
    in their natural order (a plain row-major fragment of the weights) gives a different sum for
    the A side, so the B side's order has to match the one the kernel uses."""
    rng = np.random.default_rng(1)
    W = rng.standard_normal((16, 16))
    X = rng.standard_normal((8, 16))
    a_regs, b_regs = [], []
    for lane in range(32):
        g, t = lane // 4, lane % 4
        # the kernel's A registers for its MMA j = 0 of a 16-column block (columns 4t .. 4t + 3)
        a_regs.append((W[g, 4 * t: 4 * t + 2], W[g + 8, 4 * t: 4 * t + 2], W[g, 4 * t + 2: 4 * t + 4],
                       W[g + 8, 4 * t + 2: 4 * t + 4]))
        # B in the natural order (k-slots 2t, 2t+1 = columns 2t, 2t+1)
        b_regs.append((X[g, 2 * t: 2 * t + 2], X[g, 2 * t + 8: 2 * t + 10]))
    got = _mma_16816(a_regs, b_regs)
    want = W @ X.T
    err = max(abs(got[lane][0] - want[lane // 4, 2 * (lane % 4)]) for lane in range(32))
    assert err > 1e-3
