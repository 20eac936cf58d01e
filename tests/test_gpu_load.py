"""Upload of GGUF tensors into HBM (load.Uploader, the reference's WeightLoader._roh at
ggufengine/models/common.py:83-116): the device bytes equal the file's, through many pieces and a ring
shorter than the piece count, and a matvec on the uploaded block data equals one on the same bytes
copied directly; `install` replaces a reference-style loader's _roh."""
import numpy as np
import pytest
import torch

from nemicli_terminal_b200 import load, mmvq, synth
from nemicli_terminal_b200.formats import TYPE_ID

pytestmark = pytest.mark.gpu


def _file(tmp_path):
    w = synth.blocks("Q4_K", 4096, 4096, seed=3)
    d = synth.blocks("Q6_K", 512, 1024, seed=4)
    p = tmp_path / "m.gguf"
    load.write_gguf(p, [("gate", (4096, 4096), TYPE_ID["Q4_K"], w.numpy().tobytes()),
                        ("down", (1024, 512), TYPE_ID["Q6_K"], d.numpy().tobytes()),
                        ("small", (7,), 0, np.ones(7, np.float32).tobytes())], alignment=64)
    return p, w, d


def test_upload_bytes_and_matvec(cuda, tmp_path):
    p, w, d = _file(tmp_path)
    up = load.Uploader(cuda, piece=1 << 20, buffers=3)         # 9 MB in 1 MiB pieces through 3 buffers
    with load.GGUFReader(p) as gg:
        gate = up.roh(gg, gg.tensors["gate"])
        down = up.roh(gg, gg.tensors["down"])
        small = up.roh(gg, gg.tensors["small"])
        assert gate.device.type == "cuda" and gate.dtype == torch.uint8
        assert torch.equal(gate.cpu(), w.reshape(-1)) and torch.equal(down.cpu(), d.reshape(-1))
        assert small.numel() == 28 and torch.equal(small.cpu().view(torch.float32), torch.ones(7))
        assert up.loaded_bytes == sum(t.n_bytes for t in gg.tensor_list)
    x = synth.activations(1, 4096, seed=5, device=cuda)[0]
    assert torch.equal(mmvq.mv("Q4_K", gate.view(4096, -1), x, 4096, 4096),
                       mmvq.mv("Q4_K", w.to(cuda), x, 4096, 4096))


def test_install_on_a_loader(cuda, tmp_path):
    p, w, _ = _file(tmp_path)

    class Loader:                                  # the attributes WeightLoader._roh uses
        def __init__(self, gg):
            self.gg, self.device = gg, cuda

        def _roh(self, ti, device):
            return torch.from_numpy(np.frombuffer(bytes(self.gg.tensor_bytes(ti)), np.uint8).copy())
    with load.GGUFReader(p) as gg:
        ld = Loader(gg)
        up = load.install(ld, piece=3 << 20)
        t = ld._roh(gg.tensors["gate"], cuda)
        assert t.device.type == "cuda" and torch.equal(t.cpu(), w.reshape(-1))
        c = ld._roh(gg.tensors["gate"], "cpu")     # CPU targets keep the loader's own path
        assert c.device.type == "cpu" and torch.equal(c, w.reshape(-1))
        assert up.loaded_bytes == gg.tensors["gate"].n_bytes
