"""Pretrained EDM teacher loading (train/image/main/edm/edm_unified_model.py:13-21): a release-style
pickle whose classes are not importable, wrapped in a ``torch_utils.persistence`` record whose embedded
source must never run; plain state-dict files; the DMAD generator and critic start from the teacher."""
import pickle
import sys
import types

import pytest
import torch

from dmad_b200.models.edm import EDMPrecond, load_edm_teacher, read_edm_teacher


def _small(zero=False):
    torch.manual_seed(4)
    n = EDMPrecond(16, 3, label_dim=10, model_channels=32, channel_mult=(1, 2), num_blocks=1, attn_resolutions=(8,))
    if zero:
        with torch.no_grad():
            for p in n.parameters():
                p.zero_()
    return n


def _release_pickle(net, path):
    """Pickles ``net`` as an EDM release does: a persistence record (class source embedded) under a
    module that is gone at load time; executing the record's function would set ``ran``."""
    ran = {"src": False}

    def _reconstruct_persistent_obj(meta):  # the EDM one execs meta["module_src"]
        ran["src"] = True
        raise RuntimeError("embedded source executed")

    _reconstruct_persistent_obj.__module__ = "torch_utils.persistence"
    _reconstruct_persistent_obj.__qualname__ = "_reconstruct_persistent_obj"
    mod = types.ModuleType("torch_utils.persistence")
    mod._reconstruct_persistent_obj = _reconstruct_persistent_obj
    sys.modules["torch_utils"], sys.modules["torch_utils.persistence"] = types.ModuleType("torch_utils"), mod

    class Persistent:
        def __reduce__(self):
            meta = dict(type="class", version=6, module_src="raise SystemExit('ran')", class_name="EDMPrecond",
                        state={"_parameters": net._parameters, "_buffers": net._buffers,
                               "_non_persistent_buffers_set": net._non_persistent_buffers_set,
                               "_modules": net._modules, "sigma_data": 0.5})
            return (_reconstruct_persistent_obj, (meta,))

    try:
        with open(path, "wb") as f:
            pickle.dump({"ema": Persistent(), "augment_pipe": None}, f)
    finally:
        del sys.modules["torch_utils"], sys.modules["torch_utils.persistence"]
    return ran


def test_release_pickle_reads_without_running_code(tmp_path):
    net = _small()
    ran = _release_pickle(net, str(tmp_path / "edm.pkl"))
    sd = read_edm_teacher(str(tmp_path / "edm.pkl"))
    assert not ran["src"]
    want = net.state_dict()
    assert set(sd) == set(want)
    for k in want:
        torch.testing.assert_close(sd[k], want[k], rtol=0, atol=0)
    dst = load_edm_teacher(_small(zero=True), str(tmp_path / "edm.pkl"))
    for k, v in dst.state_dict().items():
        torch.testing.assert_close(v, want[k], rtol=0, atol=0)


@pytest.mark.parametrize("fmt", ["pt", "safetensors"])
def test_state_dict_files(tmp_path, fmt):
    sd = {k: v.contiguous() for k, v in _small().state_dict().items()}
    path = str(tmp_path / f"edm.{fmt}")
    if fmt == "pt":
        torch.save({"ema": sd}, path)
    else:
        from safetensors.torch import save_file
        save_file(sd, path)
    dst = load_edm_teacher(_small(zero=True), path)
    for k, v in dst.state_dict().items():
        torch.testing.assert_close(v, sd[k], rtol=0, atol=0)
    torch.save({"model.bogus": torch.zeros(1)}, str(tmp_path / "bad.pt"))
    with pytest.raises(KeyError):
        load_edm_teacher(_small(zero=True), str(tmp_path / "bad.pt"))


def test_edm_dmad_starts_from_model_id(tmp_path):
    from dmad_b200.distill.edm_dmad import EDMDMAD, EDMDMADConfig
    from dmad_b200.models.edm import config1_unet

    torch.manual_seed(9)
    sd = {k: v.contiguous() for k, v in config1_unet(1000).state_dict().items()}
    torch.save(sd, str(tmp_path / "teacher.pt"))
    m = EDMDMAD(EDMDMADConfig(model_id=str(tmp_path / "teacher.pt"), generator_spectral_norm=False))
    got = m.generator.state_dict()
    k = next(k for k in sd if k.endswith("conv0.weight"))
    torch.testing.assert_close(got[k], sd[k], rtol=0, atol=0)
    crit = m.critic.fake_unet.state_dict()  # spectrally normed: the parametrization keeps the weight
    w = crit.get(k, crit.get(k.replace(".weight", ".parametrizations.weight.original")))
    torch.testing.assert_close(w, sd[k], rtol=0, atol=0)
