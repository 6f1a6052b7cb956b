"""CPU-side checks of the boundary: the C-ABI library loads, exports every symbol
include/b2q4nx.h declares, and its host-side logic behaves without a GPU.  The
q4nx reader's host parts are checked against the golden container."""

import ctypes

import numpy as np
import pytest

from llmnputest_b200 import _native, format as fmt
from tests.conftest import bf16_from_bits


def test_library_exports_every_header_symbol():
    syms = _native.header_symbols()
    assert len(syms) >= 10
    lib = _native.lib()
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    # and the ctypes table covers the header exactly
    assert sorted(_native.SIGNATURES) == syms


def test_version_and_status_strings():
    lib = _native.lib()
    assert lib.b2_version() == (0 << 16) | (1 << 8)
    assert lib.b2_status_string(0) == b"ok"
    assert lib.b2_status_string(-4) == b"no CUDA device"
    assert lib.b2_status_string(12345) == b"unknown status"


def test_calls_fail_cleanly_without_a_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; covered by the gpu tests")
    lib = _native.lib()
    st = lib.b2_q4_gemv(None, 1, 1, None, 1, 256, None, 32, 0, None)
    assert st == -4  # B2_ERR_NO_DEVICE: checked before any argument is touched
    assert b"device" in lib.b2_last_error_message()


def test_format_constants_match_oracle():
    from oracle import q4nx_oracle as orc
    assert (fmt.Q4_TILE_BYTES, fmt.Q8_TILE_BYTES) == (orc.Q4_TILE_BYTES, orc.Q8_TILE_BYTES) == (5120, 8704)
    assert np.array_equal(fmt.meta_index(), orc.meta_of_weight())
    t = np.arange(4096, dtype=np.uint8)
    assert np.array_equal(fmt.unpack_nibbles(t), orc.q4_codes(t))
    assert np.array_equal(fmt.to_matrix(np.arange(8192)), orc.tile_matrix(np.arange(8192)))


def test_reader_header_and_raw(container_path, golden):
    f = fmt.Q4NX(container_path)
    assert f.names() == sorted(golden["ctr_names"].tolist())
    assert "lm_head.weight" in f and "nope" not in f
    assert np.array_equal(np.frombuffer(f.raw("model.layers.0.mlp.down_proj.weight"), np.uint8),
                          golden["ctr_down_raw"])
    norm = f.tensor("model.norm.weight")  # stored as-is, no decode needed
    assert np.array_equal(norm.view(np.uint16), golden["ctr_norm"])
    # tiled shapes: 3-D (Qwen) form is self-describing, 2-D (granite) needs N or K
    assert f.tiled_shape("lm_head.weight") == (2, 4, 8704)
    assert f.tiled_shape("model.layers.0.mlp.gate_proj.weight") == (3, 2, 5120)
    assert f.tiled_shape("model.layers.0.mlp.down_proj.weight", n=64) == (2, 3, 5120)
    assert f.tiled_shape("model.layers.0.mlp.down_proj.weight", k=768) == (2, 3, 5120)
    with pytest.raises(ValueError):
        f.tiled_shape("model.layers.0.mlp.down_proj.weight")
    with pytest.raises(ValueError):
        f.tiled_shape("model.layers.0.mlp.down_proj.weight", n=128, k=768)


def test_reader_mmap_slices(container_path):
    """raw_view (mmap) equals raw(); TP slices of whole tile-rows / K-tiles are the
    stored bytes of exactly those tiles (tools/q4nx.py:170-197 layout), in the order asked."""
    f = fmt.Q4NX(container_path)
    for name in f.names():
        assert bytes(f.raw_view(name)) == f.raw(name)
    lm = np.frombuffer(f.raw("lm_head.weight"), np.uint8).reshape(2, 4, 8704)  # [n_t][k_t][tile]
    got = f.device_tiles("lm_head.weight", "cpu", tile_rows=[1]).numpy()
    assert np.array_equal(got, lm[1].reshape(-1))
    got = f.device_tiles("lm_head.weight", "cpu", tile_rows=[1, 0], k_tiles=(1, 3)).numpy()
    assert np.array_equal(got, lm[[1, 0], 1:3].reshape(-1))
    down = np.frombuffer(f.raw("model.layers.0.mlp.down_proj.weight"), np.uint8).reshape(2, 3, 5120)
    got = f.device_tiles("model.layers.0.mlp.down_proj.weight", "cpu", k_tiles=(2, 3), n=64).numpy()
    assert np.array_equal(got, down[:, 2:3].reshape(-1))
    assert len(f.tile_segments("model.layers.0.mlp.gate_proj.weight", [0, 1, 2])) == 1  # merged rows
    for bad in ({"tile_rows": [2]}, {"tile_rows": []}, {"k_tiles": (3, 3)}, {"k_tiles": (0, 5)}):
        with pytest.raises(ValueError):
            f.tile_segments("lm_head.weight", **bad)


def test_split_q4_tile_roundtrip(golden):
    t = golden["fmt_q4_tiles"][0]
    nib, d, m = fmt.split_q4_tile(t.tobytes())
    assert np.array_equal(nib, t[1024:])
    assert np.array_equal(fmt.pack_meta(d, m).view(np.uint8), t[:1024])


def test_config5_layer_entry_points_fail_cleanly_without_a_device():
    """The gated DeltaNet and gated attention entry points check the device before any
    argument, and the torch wrappers refuse host tensors (no CPU fallback)."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; covered by the gpu tests")
    lib = _native.lib()
    st = lib.b2_gated_delta_step(None, 512, None, 256, None, None, 2, None, None, None, None, None, None, 1, 1, 2,
                                 128, ctypes.c_float(1e-6), None, 256, 0, None)
    assert st == -4
    n = ctypes.c_size_t()
    assert lib.b2_gated_attn_decode_workspace_size(1, 8, 2, 256, 2048, ctypes.byref(n)) == -4
    st = lib.b2_gated_attn_decode(None, 4096, None, None, 512, None, None, None, 64, None, None, None, 1, 8, 2, 256,
                                  2048, 2048, ctypes.c_float(1e-6), None, 2048, 0, None, 0, None)
    assert st == -4
    from llmnputest_b200 import ops
    x = torch.zeros(1, 8192)
    with pytest.raises(ValueError, match="CUDA"):
        ops.gated_delta_step(x, x, x, x, x, x, x, x, x, x, 1, 2)
    with pytest.raises(ValueError, match="CUDA"):
        ops.gated_attn_decode(x, x, x, x, x, x, x, x, x, 8, 2)
