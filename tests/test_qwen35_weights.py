"""Qwen3.5 layer weights from a q4nx file (FastFlowLM names and conventions,
reference/from_q4nx.py:46-136) on CPU: the q_proj query/gate regroup is a tile-row
order and reproduces the per-head rows, the norm / A_log / conv conventions, and a
DeltaNetLayer built from the file (dense in_proj_b / in_proj_a) steps like the
oracle composition of the same file read the reference's way.  The GPU ops are the
oracle-backed shim of the host-logic tests."""

import json
import struct

import numpy as np
import pytest
import torch
from ml_dtypes import bfloat16

from llmnputest_b200.deltanet import DeltaNetLayer
from llmnputest_b200.format import Q4NX
from llmnputest_b200.qwen35 import deltanet_weights, gated_attention_weights, q_gate_tile_rows
from oracle import deltanet_oracle as dn
from oracle import q4nx_oracle as orc
from tests.test_tp_deltanet_host import DeltaOracleOps

HIDDEN, NK, NV, NQ, NKV = 256, 2, 4, 2, 1
DD, DA = 128, 256  # linear / full attention head dims
CONV = (2 * NK + NV) * DD


def _bf16_bits(a):
    return np.asarray(a, np.float32).astype(bfloat16).view(np.uint16)


@pytest.fixture(scope="module")
def qwen_file(tmp_path_factory):
    rng = np.random.default_rng(35)
    q4 = lambda rows, k: orc.synth_q4_tiles(rng, rows // 32 * (k // 256)).reshape(rows // 32, k // 256, 5120)
    L0, L1 = "model.layers.0.", "model.layers.1."
    t = {
        L0 + "linear_attn.qkv_proj.weight": ("I8", q4(CONV, HIDDEN)),
        L0 + "self_attn.gate_proj.weight": ("I8", q4(NV * DD, HIDDEN)),
        L0 + "linear_attn.ssm_beta_proj.bf16.weight": ("BF16", _bf16_bits(0.05 * rng.standard_normal((NV, HIDDEN)))),
        L0 + "linear_attn.ssm_alpha_proj.bf16.weight": ("BF16", _bf16_bits(0.05 * rng.standard_normal((NV, HIDDEN)))),
        L0 + "linear_attn.ssm_out_proj.weight": ("I8", q4(HIDDEN, NV * DD)),
        L0 + "linear_attn.ssm_conv1d.weight": ("F32", (0.5 * rng.standard_normal((4, CONV))).astype(np.float32)),
        L0 + "linear_attn.ssm_a": ("F32", -rng.uniform(0.01, 10.0, NV).astype(np.float32)),
        L0 + "linear_attn.ssm_dt.bias": ("F32", rng.standard_normal(NV).astype(np.float32)),
        L0 + "linear_attn.ssm_norm.weight": ("F32", (1 + 0.1 * rng.standard_normal(DD)).astype(np.float32)),
        L0 + "input_layernorm.weight": ("BF16", _bf16_bits(1.4 + 0.1 * rng.standard_normal(HIDDEN))),
        L1 + "self_attn.q_proj.weight": ("I8", q4(2 * NQ * DA, HIDDEN)),
        L1 + "self_attn.k_proj.weight": ("I8", q4(NKV * DA, HIDDEN)),
        L1 + "self_attn.v_proj.weight": ("I8", q4(NKV * DA, HIDDEN)),
        L1 + "self_attn.o_proj.weight": ("I8", q4(HIDDEN, NQ * DA)),
        L1 + "self_attn.q_norm.weight": ("BF16", _bf16_bits(1 + 0.1 * rng.standard_normal(DA))),
        L1 + "self_attn.k_norm.weight": ("BF16", _bf16_bits(1 + 0.1 * rng.standard_normal(DA))),
        L1 + "input_layernorm.weight": ("BF16", _bf16_bits(1.2 + 0.1 * rng.standard_normal(HIDDEN))),
    }
    header, blobs, off = {}, [], 0
    for name, (dt, arr) in t.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hj = json.dumps(header).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    path = tmp_path_factory.mktemp("q35") / "model.q4nx"
    path.write_bytes(struct.pack("<Q", len(hj)) + hj + b"".join(blobs))
    return Q4NX(path)


def test_q_gate_regroup_is_a_tile_row_order(qwen_file):
    assert q_gate_tile_rows(2) == [*range(0, 8), *range(16, 24), *range(8, 16), *range(24, 32)]
    inv = np.arange(32, dtype=np.float32)
    W = gated_attention_weights(qwen_file, 1, NQ, NKV, HIDDEN, inv, device="cpu")
    f = qwen_file
    stored_q = orc.q4_matrix(f.raw_view("model.layers.1.self_attn.q_proj.weight"), 2 * NQ * DA // 32, 1)
    got = orc.q4_matrix(W["in_proj"].numpy(), (2 * NQ + 2 * NKV) * DA // 32, 1)
    for h in range(NQ):  # transformers' per-head [q_h | gate_h] (reference/from_q4nx.py:121-126)
        assert np.array_equal(got[h * 2 * DA:h * 2 * DA + DA], stored_q[h * DA:(h + 1) * DA])
        assert np.array_equal(got[h * 2 * DA + DA:(h + 1) * 2 * DA], stored_q[(NQ + h) * DA:(NQ + h + 1) * DA])
    stored_k = orc.q4_matrix(f.raw_view("model.layers.1.self_attn.k_proj.weight"), NKV * DA // 32, 1)
    assert np.array_equal(got[2 * NQ * DA:2 * NQ * DA + NKV * DA], stored_k)
    # q/k norms: the file holds 1 + w
    qn = np.asarray(f.tensor("model.layers.1.self_attn.q_norm.weight"), np.float32)
    assert np.array_equal(W["q_norm_w"].numpy(), qn - 1.0)
    assert np.array_equal(W["o_proj"].numpy(), np.asarray(f.raw_view("model.layers.1.self_attn.o_proj.weight")))


def test_deltanet_conventions(qwen_file):
    W = deltanet_weights(qwen_file, 0, NK, NV, HIDDEN, device="cpu")
    f = qwen_file
    p = "model.layers.0.linear_attn."
    ssm_a = np.asarray(f.tensor(p + "ssm_a"), np.float32)
    np.testing.assert_allclose(-np.exp(W["A_log"].numpy()), ssm_a, rtol=1e-6)
    assert np.array_equal(W["conv_w"].numpy(), np.asarray(f.tensor(p + "ssm_conv1d.weight")).T)
    assert W["conv_w"].shape == (CONV, 4) and W["conv_w"].is_contiguous()
    assert W["ba_dense"].shape == (2 * NV, HIDDEN)


def test_deltanet_layer_from_file_steps_like_reference(qwen_file):
    """Two steps of a DeltaNetLayer built from the file, against the reference's reading of
    the same file: dense dequantised matrices, A_log = log(-ssm_a), conv transposed."""
    W = deltanet_weights(qwen_file, 0, NK, NV, HIDDEN, device="cpu")
    layer = DeltaNetLayer(HIDDEN, NK, NV, 2, device="cpu", weights=W, ops_impl=DeltaOracleOps())
    f = qwen_file
    p = "model.layers.0."
    qkv_m = orc.q4_matrix(f.raw_view(p + "linear_attn.qkv_proj.weight"), CONV // 32, 1)
    z_m = orc.q4_matrix(f.raw_view(p + "self_attn.gate_proj.weight"), NV * DD // 32, 1)
    b_m = np.asarray(f.tensor(p + "linear_attn.ssm_beta_proj.bf16.weight"), np.float32)
    a_m = np.asarray(f.tensor(p + "linear_attn.ssm_alpha_proj.bf16.weight"), np.float32)
    out_raw = f.raw_view(p + "linear_attn.ssm_out_proj.weight")
    norm_in = np.asarray(f.tensor(p + "input_layernorm.weight"), np.float32)
    conv_w = np.asarray(f.tensor(p + "linear_attn.ssm_conv1d.weight"), np.float32).T
    a_log = np.log(-np.asarray(f.tensor(p + "linear_attn.ssm_a"), np.float32))
    dt_b = np.asarray(f.tensor(p + "linear_attn.ssm_dt.bias"), np.float32)
    nrm = np.asarray(f.tensor(p + "linear_attn.ssm_norm.weight"), np.float32)
    r_conv = np.zeros((2, CONV, 4), np.float32)
    r_state = np.zeros((2, NV, DD, DD))
    rng = np.random.default_rng(1)
    for t in range(2):
        x = rng.standard_normal((2, HIDDEN)).astype(np.float32)
        resid = torch.from_numpy(x.copy())
        layer.step(resid)
        xn = orc.rmsnorm(x, norm_in, 1e-6).astype(bfloat16).astype(np.float32)
        o, r_conv, r_state = dn.gated_delta_step(xn @ qkv_m.T, xn @ z_m.T, xn @ b_m.T, xn @ a_m.T, r_conv, conv_w,
                                                 a_log, dt_b, nrm, r_state, NK, NV, DD, DD)
        ref = x + orc.gemv_q4(out_raw, o.astype(bfloat16).astype(np.float32), HIDDEN // 32, NV * DD // 256)
        cos, rel = orc.compare(resid.numpy(), ref)
        assert cos >= 0.99999 and rel <= 1e-3, (t, cos, rel)
