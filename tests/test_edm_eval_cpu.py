"""The EDM family's generator EMAs: saved in checkpoints (a resume restores them), exported per checkpoint
under the reference's file names, and evaluated by the checkpoint-folder FID evaluator (one-step samples
with cycling labels, the caller's detector, results in stats.json)."""
import json
import os

import numpy as np
import torch

CFG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "configs", "edm_imagenet64_dmad.yaml")


class _Det(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.lin = torch.nn.Linear(3 * 64 * 64, 8)

    def forward(self, x, return_features: bool = True):
        return torch.tanh(self.lin(x.float().flatten(1) / 255.0))


def test_ema_checkpoint_export_and_folder_fid(tmp_path):
    from dmad_b200.cli.train import main as train
    from dmad_b200.models.edm import config1_unet
    from dmad_b200.tools.edm_eval_folder import ema_weight_files, main as evaluate, one_step_samples

    out = str(tmp_path / "edm")
    train(["--config", CFG, f"training.output_dir={out}", "training.max_iters=2", "training.save_every=1",
           "training.log_every=1"])
    ck1, ck2 = (os.path.join(out, f"checkpoint-{i:09d}") for i in (1, 2))
    assert [m for m, _ in ema_weight_files(ck2)] == ["fid", "fid_ema_8000", "fid_ema_16000"]
    shared = torch.load(os.path.join(ck2, "shared.pt"), map_location="cpu", weights_only=False)
    ema_keys = [k for k in shared if k.startswith("module/ema_")]
    assert ema_keys == ["module/ema_1000", "module/ema_8000", "module/ema_16000"]
    assert shared["ema_state"]["step_count"] == 2
    exported = torch.load(os.path.join(ck2, "pytorch_model_ema.bin"), map_location="cpu")
    assert not any(".sn_" in k for k in exported)  # the generator's spectral norm is folded into the weights
    # the exported file loads into a plain config-1 network that computes what the saved EMA computes
    net = config1_unet(1000)
    net.load_state_dict(exported)
    # the EMA is its own state (not the generator's), and loading a checkpoint restores it
    assert any(not torch.equal(v, shared["module/generator"][k]) for k, v in shared["module/ema_1000"].items())
    from dmad_b200.train.registry import build_model
    adapter = build_model({"model": {"family": "edm_dmad"}}, "cpu", 0)
    adapter.load_state_dicts(shared, None)
    assert adapter.model.step_count == 2
    for k, v in adapter.model.emas[1000.0].state_dict().items():
        torch.testing.assert_close(v, shared["module/ema_1000"][k])
    ema_net = adapter.model.emas[1000.0].eval()
    x, sig, lab = torch.randn(2, 3, 64, 64) * 80, torch.full((2,), 80.0), torch.eye(1000)[[3, 7]]
    with torch.no_grad():
        torch.testing.assert_close(net.eval()(x, sig, lab), ema_net(x, sig, lab), rtol=1e-4, atol=1e-4)
    train(["--config", CFG, f"training.output_dir={out}", "training.max_iters=3", "training.save_every=1",
           "training.log_every=1"])

    # one-step samples: deterministic for the seed, labels i mod label_dim
    a = torch.cat(list(one_step_samples(net.eval(), 5, 4, 10, 1000, 64, 80.0, "cpu")))
    b = torch.cat(list(one_step_samples(net.eval(), 5, 4, 10, 1000, 64, 80.0, "cpu")))
    assert a.shape == (5, 3, 64, 64) and a.dtype == torch.uint8 and torch.equal(a, b)

    det = str(tmp_path / "det.pt")
    torch.manual_seed(0)
    torch.jit.script(_Det()).save(det)
    rng = np.random.RandomState(0)
    feats = rng.randn(40, 8) * 0.3
    ref = str(tmp_path / "ref.npz")
    np.savez(ref, mu=feats.mean(0), sigma=np.cov(feats, rowvar=False))
    stats = evaluate(["--folder", out, "--ref", ref, "--detector", det, "--num", "6", "--batch", "4",
                      "--device", "cpu", "--run-once"])
    assert sorted(stats) == ["checkpoint-000000001", "checkpoint-000000002", "checkpoint-000000003"]
    assert all(np.isfinite(v["fid"]) and np.isfinite(v["fid_ema_16000"]) and v["iteration"] == int(k[-9:])
               for k, v in stats.items())
    on_disk = json.load(open(os.path.join(out, "stats.json")))
    assert on_disk.keys() == stats.keys()
    # already evaluated checkpoints are skipped on the next pass
    assert evaluate(["--folder", out, "--ref", ref, "--detector", det, "--num", "6", "--batch", "4",
                     "--device", "cpu", "--run-once"]) == on_disk
