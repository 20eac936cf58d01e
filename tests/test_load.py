"""GGUF reader / writer of the load side (CPU): round trips, piecewise reads, and refusal of malformed
files (the checks of the reference's reader, ggufengine/gguf.py:203-271)."""
import struct

import numpy as np
import pytest

from nemicli_terminal_b200 import load, synth
from nemicli_terminal_b200.formats import TYPE_ID


def _tensors():
    q4k = synth.blocks("Q4_K", 64, 512, seed=1).numpy().tobytes()
    q6k = synth.blocks("Q6_K", 8, 256, seed=2).numpy().tobytes()
    f32 = np.arange(10, dtype=np.float32).tobytes()
    return [("blk.0.ffn_gate.weight", (512, 64), TYPE_ID["Q4_K"], q4k),
            ("blk.0.ffn_down.weight", (256, 8), TYPE_ID["Q6_K"], q6k),
            ("blk.0.norm.weight", (10,), 0, f32)]


def test_round_trip(tmp_path):
    p = tmp_path / "m.gguf"
    load.write_gguf(p, _tensors(), {"general.architecture": "llama", "llama.block_count": 1, "x.eps": 1e-5})
    with load.GGUFReader(p) as gg:
        assert gg.metadata["general.architecture"] == "llama" and gg.metadata["llama.block_count"] == 1
        assert [t.name for t in gg.tensor_list] == [t[0] for t in _tensors()]
        for name, dims, t, data in _tensors():
            ti = gg.tensors[name]
            assert ti.dims == dims and ti.ggml_type == t and ti.n_bytes == len(data)
            assert ti.offset % gg.alignment == 0 and ti.shape == tuple(reversed(dims))
            assert bytes(gg.tensor_bytes(ti)) == data
            buf = np.zeros(1000, dtype=np.uint8)        # pieces of 1000 bytes, the last one short
            got = bytearray()
            for start in range(0, ti.n_bytes, 1000):
                n = gg.read_into(ti, buf, start)
                got += buf[:n].tobytes()
            assert bytes(got) == data


def test_alignment_and_refusals(tmp_path):
    p = tmp_path / "a.gguf"
    load.write_gguf(p, _tensors(), alignment=256)
    with load.GGUFReader(p) as gg:
        assert gg.alignment == 256 and all(t.offset % 256 == 0 for t in gg.tensor_list)
    raw = bytearray(p.read_bytes())
    bad = tmp_path / "b.gguf"
    bad.write_bytes(b"GGUX" + raw[4:])
    with pytest.raises(load.GGUFError):
        load.GGUFReader(bad)
    bad.write_bytes(raw[:len(raw) - 100])                  # last tensor runs past the end
    with pytest.raises(load.GGUFError):
        load.GGUFReader(bad)
    bad.write_bytes(raw[:40])                              # header cut short
    with pytest.raises(load.GGUFError):
        load.GGUFReader(bad)
    big = bytearray(raw)
    big[8:16] = struct.pack("<Q", 1 << 40)                 # tensor count beyond the limit
    bad.write_bytes(big)
    with pytest.raises(load.GGUFError):
        load.GGUFReader(bad)
    with pytest.raises(ValueError):
        load.write_gguf(bad, [("t", (300,), TYPE_ID["Q4_K"], b"\0" * 144)])   # not whole superblocks
    with load.GGUFReader(p) as gg:
        with pytest.raises(load.GGUFError):
            gg.read_into(gg.tensor_list[0], np.zeros(8, np.uint8), gg.tensor_list[0].n_bytes + 1)


def test_uploader_needs_cuda():
    with pytest.raises(ValueError):
        load.Uploader("cpu")
