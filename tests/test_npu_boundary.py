"""The reference-facing plugin surface (llmnputest_b200.npu mirrors reference/npu.py)."""

import numpy as np
import pytest
import torch
from ml_dtypes import bfloat16

from llmnputest_b200 import format as fmt
from llmnputest_b200 import npu
from oracle import q4nx_oracle as orc


def test_design_meta_buffers():
    m = npu._with_buffers(npu.DESIGNS["lm_head"])
    assert m["buffers"] == [7760 * 4 * 8704, 1024 * 2, 248320 * 4]  # 270 MB of q8 tiles
    m = npu._with_buffers(npu.DESIGNS["granite_lm_head"])
    assert m["buffers"][0] == 3136 * 10 * 5120
    with pytest.raises(ValueError):
        npu._with_buffers({"kind": "q4_gemv", "n_rows": 100, "k": 256})


def test_no_cpu_fallback_without_gpu():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(SystemExit):
        npu.NpuDesign("lm_head")


@pytest.mark.gpu
def test_design_upload_run_download():
    rng = np.random.default_rng(8)
    n_t, k_t = 130, 4
    w = orc.synth_q8_tiles(rng, n_t * k_t)
    x = rng.standard_normal(1024).astype(np.float32)
    d = npu.NpuDesign("lm_head", meta={"kind": "q8_gemv", "n_rows": n_t * 32, "k": 1024})
    d.upload(0, w)
    d.upload(1, npu.bf16_host(x))
    d.run()
    y = d.download(2, np.float32, n_t * 32)
    cos, rel = orc.compare(y, orc.gemv_q8(w, x.astype(bfloat16), n_t, k_t))
    assert cos > 0.9999999 and rel < 1e-4
    d.close()


@pytest.mark.gpu
def test_lm_head_module_on_container(container_path, golden):
    """NpuLmHead over the golden .q4nx: decode (1 position) and prefill (5 positions), both on the GPU."""
    f = fmt.Q4NX(container_path)

    class Model:
        lm_head = torch.nn.Linear(1024, 64, bias=False)

    model = Model()
    head = npu.NpuLmHead(model.lm_head, meta={"kind": "q8_gemv", "n_rows": 64, "k": 1024})
    head.load_weights(f.raw("lm_head.weight"))
    w = golden["ctr_lm_head_f32"]  # the reference's Q4NX.tensor() of the same bytes
    rng = np.random.default_rng(1)
    for positions in (1, 5):
        h = torch.from_numpy(rng.standard_normal((1, positions, 1024)).astype(np.float32))
        y = head(h)
        assert y.shape == (1, positions, 64) and y.device == h.device and y.dtype == h.dtype
        xb = h.numpy().reshape(positions, 1024).astype(bfloat16).astype(np.float32)
        ref = xb @ w.T
        cos, rel = orc.compare(y.numpy().reshape(positions, 64), ref)
        assert cos > 0.9999999 and rel < 1e-4
    assert head.npu_calls == 2 and head.cpu_calls == 0 and head.design.calls == 2


@pytest.mark.gpu
def test_attach_lm_head(container_path, monkeypatch):
    f = fmt.Q4NX(container_path)
    monkeypatch.setitem(npu.DESIGNS, "lm_head", {"kind": "q8_gemv", "n_rows": 64, "k": 1024})

    class Model:
        lm_head = torch.nn.Linear(1024, 64, bias=False)

    m = Model()
    head = npu.attach_lm_head(m, f)
    assert m.lm_head is head and head.n_rows == 64 and head.k == 1024


@pytest.mark.gpu
def test_reader_upload_through_pinned_staging(container_path):
    """Chunked pinned-staging uploads land the stored bytes on the GPU unchanged: whole
    tensors and TP slices, with chunks smaller than, equal to and larger than a segment."""
    import torch
    f = fmt.Q4NX(container_path)
    lm = np.frombuffer(f.raw("lm_head.weight"), np.uint8).reshape(2, 4, 8704)
    for chunk in (1000, 8704, 1 << 20):
        t = f.device_tiles("lm_head.weight", chunk_bytes=chunk)
        assert t.is_cuda and np.array_equal(t.cpu().numpy(), lm.reshape(-1))
        t = f.device_tiles("lm_head.weight", tile_rows=[1, 0], k_tiles=(1, 4), chunk_bytes=chunk)
        assert np.array_equal(t.cpu().numpy(), lm[[1, 0], 1:4].reshape(-1))
    gate = f.device_tiles("model.layers.0.mlp.gate_proj.weight", chunk_bytes=4096)
    assert np.array_equal(gate.cpu().numpy(), np.frombuffer(f.raw("model.layers.0.mlp.gate_proj.weight"), np.uint8))
    torch.cuda.synchronize()


@pytest.mark.gpu
def test_reader_decodes_on_gpu(container_path, golden):
    """Q4NX.tensor() (GPU decode) equals the reference reader's float32 output bit for bit."""
    f = fmt.Q4NX(container_path)
    assert np.array_equal(f.tensor("lm_head.weight"), golden["ctr_lm_head_f32"])
    assert np.array_equal(f.tensor("model.layers.0.mlp.gate_proj.weight"), golden["ctr_gate_f32"])
    assert np.array_equal(f.tensor("model.layers.0.mlp.gate_proj.weight", (80, 300)), golden["ctr_gate_f32_trim"])
    t = golden["fmt_q4_tiles"][0]
    nib, d, m = fmt.split_q4_tile(t.tobytes())
    assert np.array_equal(fmt.dequant_q4(nib, d, m).view(np.uint16), golden["fmt_q4_dequant_bf16"][0])
    assert np.array_equal(fmt.dequant_q8(golden["fmt_q8_tiles"][0].tobytes()).view(np.uint16),
                          golden["fmt_q8_dequant_bf16"][0])
