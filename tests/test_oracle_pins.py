"""Pin the CPU oracle to rusty-engine's own known-answer tests before trusting it.

Each test restates one reference test (inputs and expected values read from the Rust test
source; file:line given per test).  The Rust crate cannot be built here (no cargo), so these
known answers are the oracle's anchor.
"""
import math
import struct

import numpy as np
import pytest

from oracle import oracle as O

EPS = 1e-5  # src/moe.rs:623


def f32(x):
    return struct.unpack("<f", struct.pack("<f", x))[0]


# ---- src/quant.rs tests -----------------------------------------------------------------
def test_f16_known_values():  # src/quant.rs:459-471
    assert O.f16_to_f32(0x3C00) == 1.0
    assert O.f16_to_f32(0x4000) == 2.0
    assert O.f16_to_f32(0x3800) == 0.5
    assert O.f16_to_f32(0x0000) == 0.0
    assert O.f16_to_f32(0xC000) == -2.0
    assert math.isinf(O.f16_to_f32(0x7C00))
    assert struct.pack("<f", O.f16_to_f32(0x8000)) == struct.pack("<f", -0.0)
    assert O.f16_to_f32(0x0001) == 2.0 ** -24
    assert O.f16_to_f32(0x03FF) == 1023.0 * 2.0 ** -24
    assert math.isnan(O.f16_to_f32(0x7E00))
    assert math.isnan(O.f16_to_f32(0xFE00))


def test_f16_bit_exact_against_f64_reference():  # src/quant.rs:475-499, all 65536 patterns
    got = O.f16_to_f32_all()
    h = np.arange(65536, dtype=np.uint32)
    sign = np.where((h >> 15) & 1, -1.0, 1.0)
    exp = ((h >> 10) & 0x1F).astype(np.int64)
    frac = (h & 0x3FF).astype(np.float64)
    with np.errstate(invalid="ignore"):
        v = np.where(exp == 0, frac / 1024.0 * 2.0 ** -14, (1.0 + frac / 1024.0) * np.power(2.0, exp - 15))
        v = np.where((exp == 31) & (frac == 0), np.inf, v)
        v = np.where((exp == 31) & (frac != 0), np.nan, v)
    want = (sign * v).astype(np.float32)
    nan = np.isnan(want)
    assert np.all(np.isnan(got[nan]))
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))
    # and the hardware widening the GPU kernels use is the same map (numpy's f16 is IEEE)
    hw = h.astype(np.uint16).view(np.float16).astype(np.float32)
    assert np.array_equal(got[~nan].view(np.uint32), hw[~nan].view(np.uint32))


def test_block_sizes_match_ggml():  # src/quant.rs:501-545
    assert O.block_info(2) == (32, 18)
    assert O.block_info(8) == (32, 34)
    assert O.block_info(6) == (32, 22)
    assert O.block_info(12) == (256, 144)
    assert O.block_info(13) == (256, 176)
    assert O.block_info(14) == (256, 210)
    assert O.block_info(999) is None


def test_bytes_for_numel_block_math():  # src/quant.rs:547-552
    assert O.bytes_for_numel(2, 64) == 36
    assert O.bytes_for_numel(0, 10) == 40
    assert O.bytes_for_numel(2, 33) is None


def _one():
    return bytes([0x00, 0x3C])  # f16 1.0 little-endian


def test_q4_0_split_half_and_offset():  # src/quant.rs:554-568
    blk = bytearray(18)
    blk[0:2] = _one()
    blk[2] = 0x0F
    out = O.dequant(2, bytes(blk))
    assert len(out) == 32
    assert out[0] == 7.0 and out[16] == -8.0 and out[1] == -8.0 and out[31] == -8.0


def test_q4_0_all_zero_nibbles_minus_eight():  # src/quant.rs:570-576
    blk = bytearray(18)
    blk[0:2] = _one()
    assert np.all(O.dequant(2, bytes(blk)) == -8.0)


def test_q8_0_signed_values():  # src/quant.rs:578-589
    blk = bytearray(34)
    blk[0:2] = _one()
    blk[2], blk[3] = 0x7F, 0xFF
    out = O.dequant(8, bytes(blk))
    assert len(out) == 32 and out[0] == 127.0 and out[1] == -1.0


def test_q5_0_values_and_5th_bit():  # src/quant.rs:591-616
    blk = bytearray(22)
    blk[0:2] = _one()
    blk[6:22] = b"\x11" * 16
    out = O.dequant(6, bytes(blk))
    assert len(out) == 32 and np.all(out == -15.0)
    b2 = bytearray(22)
    b2[0:2] = _one()
    b2[2:6] = struct.pack("<I", 1)
    out2 = O.dequant(6, bytes(b2))
    assert out2[0] == 0.0 and out2[16] == -16.0
    b3 = bytearray(22)
    b3[0:2] = _one()
    b3[6] = 0xF0
    out3 = O.dequant(6, bytes(b3))
    assert out3[0] == -16.0 and out3[16] == -1.0


def test_dequant_dispatch_lengths():  # src/quant.rs:618-630
    with pytest.raises(O.OracleError):
        O.dequant(2, bytes(17))
    with pytest.raises(O.OracleError):
        O.dequant(6, bytes(21))
    assert len(O.dequant(6, bytes(22))) == 32
    with pytest.raises(O.OracleError):
        O.dequant(12, bytes(143))
    with pytest.raises(O.OracleError):
        O.dequant(99, bytes(8))
    ok = bytearray(18)
    ok[0:2] = _one()
    assert len(O.dequant(2, bytes(ok))) == 32
    assert len(O.dequant(12, bytes(144))) == 256


def test_q4_k_zero_block_all_zero():  # src/quant.rs:632-640
    b = bytearray(144)
    b[0:2] = _one()
    out = O.dequant(12, bytes(b))
    assert len(out) == 256 and np.all(out == 0.0)


def test_q4_k_uniform_scale_and_min():  # src/quant.rs:642-656
    b = bytearray(144)
    b[0:2] = _one()
    b[2:4] = _one()
    b[4] = 2
    b[8] = 1
    b[16:144] = b"\x03" * 128
    out = O.dequant(12, bytes(b))
    assert abs(out[0] - 5.0) < 1e-5 and abs(out[31] - 5.0) < 1e-5
    assert out[32] == 0.0


def test_q5_k_low_group():  # src/quant.rs:658-668
    b = bytearray(176)
    b[0:2] = _one()
    b[4] = 1
    b[48:176] = b"\x03" * 128
    out = O.dequant(13, bytes(b))
    assert len(out) == 256 and abs(out[0] - 3.0) < 1e-5


def test_q6_k_signed_zero_bias():  # src/quant.rs:670-678
    b = bytearray(210)
    b[208:210] = _one()
    b[192:208] = b"\x01" * 16
    out = O.dequant(14, bytes(b))
    assert len(out) == 256 and np.all(np.abs(out + 32.0) < 1e-5)


def test_dequant_f32_f16_bf16():  # src/quant.rs:680-728
    assert list(O.dequant(0, struct.pack("<3f", 1.5, -2.0, 0.125))) == [1.5, -2.0, 0.125]
    assert list(O.dequant(1, struct.pack("<3H", 0x3C00, 0x4000, 0xCC00))) == [1.0, 2.0, -16.0]
    assert list(O.dequant(30, struct.pack("<4H", 0x3F80, 0x3F00, 0xC000, 0x4452))) == [1.0, 0.5, -2.0, 840.0]
    with pytest.raises(O.OracleError, match="BF16 data len 3 not a multiple of 2"):
        O.dequant(30, bytes(3))
    with pytest.raises(O.OracleError, match="F32"):
        O.dequant(0, bytes(3))


# ---- src/moe.rs tests -------------------------------------------------------------------
def test_softmax_sums_to_one():  # src/moe.rs:625-630
    assert abs(sum(O.softmax([1.0, 2.0, 3.0])) - 1.0) < EPS


def test_top_k_picks_largest_and_renormalizes():  # src/moe.rs:632-641
    s = O.top_k([0.1, 0.9, 0.2, 0.8], 2)
    assert [e[0] for e in s] == [1, 3]
    assert abs(sum(e[1] for e in s) - 1.0) < EPS


def test_top_k_clamps_when_k_exceeds_experts():  # src/moe.rs:643-646
    assert len(O.top_k([0.5, 0.4], 8)) == 2


def test_sigmoid_silu_basics():  # src/moe.rs:648-654
    assert abs(O.sigmoid(0.0) - 0.5) < EPS
    assert O.sigmoid(10.0) > 0.999
    assert abs(O.silu(0.0)) < EPS
    assert abs(O.silu(1.0) - 1.0 / (1.0 + math.exp(-1.0))) < EPS


def test_sigmoid_router_renormalizes_to_one():  # src/moe.rs:656-663
    s = O.top_k_sigmoid([1.0, 5.0, 2.0, 4.0], 2)
    assert [e[0] for e in s] == [1, 3]
    assert abs(sum(e[1] for e in s) - 1.0) < EPS


def test_route_dispatches_by_gate():  # src/moe.rs:665-673
    assert [e[0] for e in O.route([0.0, 3.0, 1.0, 2.0], 1, 2)] == [1, 3]


def test_route_group_restricts_to_best_group():  # src/moe.rs:675-686
    s = O.route_grouped([0.0, 0.0, 0.0, 5.0, 4.0, 3.0], [], 2, 2, 1, noaux=False)
    assert len(s) == 2 and all(3 <= e[0] <= 5 for e in s)
    assert abs(sum(e[1] for e in s) - 1.0) < EPS


def test_route_noaux_tc_uses_top2_group_score_not_group_sum():  # src/moe.rs:688-703
    logits = [5.0, 2.0, -9.0, -9.0, 0.0, 0.0, 0.0, 0.0]
    noaux = O.route_grouped(logits, [], 2, 1, 1, noaux=True)
    assert noaux[0][0] == 0 and abs(noaux[0][1] - 1.0) < EPS
    lite = O.route_grouped(logits, [], 2, 1, 1, noaux=False)
    assert 4 <= lite[0][0] <= 7


def test_route_noaux_tc_renormalizes_top_k():  # src/moe.rs:705-714
    s = O.route_grouped([5.0, 2.0, -9.0, -9.0, 0.0, 0.0, 0.0, 0.0], [], 2, 2, 1, noaux=True)
    assert [e[0] for e in s] == [0, 1]
    assert abs(sum(e[1] for e in s) - 1.0) < EPS


def test_route_noaux_tc_empty_input():  # src/moe.rs:716-719
    assert O.route_grouped([], [], 2, 1, 1, noaux=True) == []


def test_matvec_identity_and_sum():  # src/moe.rs:721-728
    assert list(O.matvec([1.0, 0.0, 0.0, 1.0], 2, 2, [3.0, 4.0])) == [3.0, 4.0]
    assert list(O.matvec([1.0, 1.0], 1, 2, [3.0, 4.0])) == [7.0]


def test_expert_ffn_pipeline():  # src/moe.rs:740-750
    id2 = [1.0, 0.0, 0.0, 1.0]
    out = O.expert_ffn([1.0, 0.0], id2, id2, id2, 2, 2)
    assert abs(out[0] - O.silu(1.0)) < EPS and abs(out[1]) < EPS


def _id_expert(scale):  # src/moe.rs:765-771
    return ([1.0, 0.0, 0.0, 1.0], [1.0, 0.0, 0.0, 1.0], [scale, 0.0, 0.0, scale])


def test_moe_layer_routes_to_best_expert():  # src/moe.rs:773-786
    out = O.moe_layer_forward([1.0, 0.0], [0.0, 0.0, 10.0, 0.0], 2, [_id_expert(1.0), _id_expert(2.0)], None, 2,
                              0, 1)
    assert abs(out[0] - 2.0 * O.silu(1.0)) < EPS and abs(out[1]) < EPS


def test_moe_layer_adds_shared_expert():  # src/moe.rs:788-801
    ie = _id_expert(1.0)
    out = O.moe_layer_forward([1.0, 0.0], [10.0, 0.0, 0.0, 0.0], 2, [ie, ie], ie, 2, 1, 1)
    assert abs(out[0] - 2.0 * O.silu(1.0)) < EPS and abs(out[1]) < EPS


def test_cached_fixture_forward():  # src/moe.rs:478-521 (resident path of the cached fixture)
    router_w = [0.1, 0.2, -0.3, 0.4, -0.2, 0.9]
    mk = lambda tag: ([tag, 0.5, -0.5, tag, 0.25, -0.25, tag, 0.75], [1.0, 0.5, 0.5, 1.0, 0.25, 0.75, 0.5, 1.0],
                      [0.5, -0.5, tag, 0.25, 0.75, -0.25, 1.0, tag])
    experts = [mk(0.1), mk(0.4), mk(0.9)]
    hidden = [0.3, -0.7]
    out = O.moe_layer_forward(hidden, router_w, 3, experts, None, 4, 0, 1)
    # router logits: [0.1*.3+0.2*-.7, -.3*.3+.4*-.7, -.2*.3+.9*-.7] -> expert 0 wins (top-1, weight 1)
    want = O.expert_ffn(hidden, *experts[0], 2, 4)
    assert np.allclose(out, want, atol=1e-6)


# ---- src/kernel.rs fused-vs-dequant pins (k_blocks fixture, src/kernel.rs:2369-2391) --------
def k_blocks(kind: int, nb: int) -> bytes:
    nbytes = {0: 144, 1: 176, 2: 210}[kind]
    a = bytearray(nb * nbytes)
    for bi in range(nb):
        blk = memoryview(a)[bi * nbytes:(bi + 1) * nbytes]
        if kind != 2:
            blk[0], blk[1], blk[2], blk[3] = 0x00, 0x3C, 0x00, 0x3C
        else:
            blk[nbytes - 2], blk[nbytes - 1] = 0x00, 0x3C
        for j in range(nbytes - 4):
            blk[4 + j] = (bi * 91 + j * 7) % 251
    return bytes(a)


@pytest.mark.parametrize("kind,t", [(0, 12), (1, 13), (2, 14)])
def test_pooled_matmul_matches_rowwise_exact(kind, t):
    """matmul_matches_rowwise_matvec (src/kernel.rs:2534-2585), tolerance 1e-2*(1+|p|)."""
    O.pool_init(4)
    m, n, rows = 3, 512, 3
    w = np.frombuffer(k_blocks(kind, m * n // 256), dtype=np.uint8)
    x = (((np.arange(rows * n) * 5) % 11).astype(np.float32) * np.float32(0.1) - np.float32(0.5)).astype(np.float32)
    got = O.qmat_matmul(t, w, m, n, x.reshape(rows, n), rows)
    deq = O.dequant(t, w.tobytes()).reshape(m, n)
    want = np.stack([O.matvec(deq, m, n, x[r * n:(r + 1) * n]) for r in range(rows)])
    assert np.all(np.abs(got - want) <= 1e-2 * (1.0 + np.abs(got)))
