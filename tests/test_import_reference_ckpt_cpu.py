"""Importing a reference-layout DCP checkpoint (torch DCP directory, ``net_ema.`` prefix, spectral norm
stored as torch parametrizations) into this package's WanModel, and the SN-folded release file."""
import os

import pytest
import torch


def _model(sn):
    from dmad_b200.models.wan import WanConfig, WanModel

    torch.manual_seed(0)
    m = WanModel(WanConfig(dim=128, ffn_dim=256, num_heads=2, num_layers=2, text_dim=32, freq_dim=64))
    torch.nn.init.normal_(m.head.head.weight, std=0.05)
    if sn:
        m.enable_spectral_norm(range(2), power_iters=5)
    return m.eval()


def _to_reference_layout(sd, prefix="net_ema."):
    """This package's keys -> the reference's parametrization keys (what its DCP directory holds)."""
    layers = {k[: -len(".sn_u")] for k in sd if k.endswith(".sn_u")}
    out = {}
    for k, v in sd.items():
        base, leaf = k.rsplit(".", 1)
        if base in layers and leaf != "bias":
            name = {"weight": "original", "sn_u": "0._u", "sn_v": "0._v", "sn_gain": "1.gain"}.get(leaf)
            if name is None:
                continue
            out[f"{prefix}{base}.parametrizations.weight.{name}"] = v.clone()
        else:
            out[prefix + k] = v.clone()
    out["net.unrelated"] = torch.zeros(1)  # other sub-modules of the distillation model are ignored
    return out


def test_import_dcp_with_spectral_norm_and_release(tmp_path):
    import torch.distributed.checkpoint as dcp

    from dmad_b200.tools.import_reference_checkpoint import fold_spectral_norm, read_dcp, to_package_keys

    src = _model(sn=True)
    ref_sd = _to_reference_layout(src.state_dict())
    dcp.save(ref_sd, checkpoint_id=str(tmp_path / "model"), no_dist=True)
    sd = to_package_keys(read_dcp(str(tmp_path / "model")), "net_ema.")
    dst = _model(sn=True)
    with torch.no_grad():
        for p in dst.parameters():
            p.zero_()
    dst.load_state_dict(sd)
    for (k, a), b in zip(src.state_dict().items(), dst.state_dict().values()):
        assert torch.equal(a, b), k
    # the release fold (one power iteration from the stored u, as the reference's converter) equals this
    # package's own fold of the same layers (SegLinear.folded_weight, used by export_release)
    from dmad_b200.models.layers import SegLinear

    plain = _model(sn=False)
    plain.load_state_dict(fold_spectral_norm(sd))
    n = 0
    for name, mod in dst.named_modules():
        if isinstance(mod, SegLinear) and mod.sn_enabled:
            torch.testing.assert_close(plain.get_submodule(name).weight.float(), mod.folded_weight().float(),
                                       rtol=1e-5, atol=1e-6)
            n += 1
    assert n == 14


def test_cli_writes_state_and_release(tmp_path):
    import torch.distributed.checkpoint as dcp

    from dmad_b200.tools.import_reference_checkpoint import main

    dcp.save(_to_reference_layout(_model(sn=False).state_dict()), checkpoint_id=str(tmp_path / "model"), no_dist=True)
    main([str(tmp_path / "model"), str(tmp_path / "out.pt"), "--release", str(tmp_path / "rel.pth")])
    rel = torch.load(tmp_path / "rel.pth")
    assert all(k.startswith("net.") for k in rel) and rel["net.head.head.weight"].dtype == torch.bfloat16
    assert os.path.getsize(tmp_path / "out.pt") > 0


@pytest.mark.parametrize("fmt", ["release_pth", "plain_pt", "safetensors", "dcp"])
def test_wan_dmad_starts_from_teacher_ckpt(tmp_path, fmt):
    """``teacher_ckpt``: student, critic backbone (and the teacher, when kept) start from the checkpoint
    in any of the formats the reference's runs produce (rcm :197-251)."""
    from dmad_b200.distill.wan_dmad import WanDMAD, WanDMADConfig
    from dmad_b200.models.wan import WanConfig, WanModel

    cfg = WanConfig(dim=64, ffn_dim=128, num_heads=1, num_layers=2, text_dim=16)
    torch.manual_seed(11)
    src = WanModel(cfg)
    sd = {k: v.clone().contiguous() for k, v in src.state_dict().items()}
    if fmt == "release_pth":
        path = str(tmp_path / "teacher.pth")
        torch.save({f"net.{k}": v for k, v in sd.items()}, path)
    elif fmt == "plain_pt":
        path = str(tmp_path / "teacher.pt")
        torch.save({"model": sd}, path)
    elif fmt == "safetensors":
        from safetensors.torch import save_file
        path = str(tmp_path / "teacher.safetensors")
        save_file(sd, path)
    else:
        import torch.distributed.checkpoint as dcp
        path = str(tmp_path / "dcp")
        dcp.save({f"net_ema.{k}": v for k, v in sd.items()}, checkpoint_id=path, no_dist=True)
    m = WanDMAD(WanDMADConfig(net=cfg, teacher_ckpt=path, critic_mode="dmd", critic_spectral_norm=False,
                              generator_spectral_norm=False), device="cpu", dtype=torch.float32)
    for net in (m.net, m.net_fake_score, m.net_teacher):
        got = net.state_dict()
        for k in ("patch_embedding.weight", "blocks.1.self_attn.k.weight", "head.head.bias"):
            if k in sd:
                torch.testing.assert_close(got[k], sd[k], rtol=0, atol=0)
    with pytest.raises(KeyError):
        torch.save({"net.patch_embedding.weight": sd["patch_embedding.weight"]}, str(tmp_path / "bad.pth"))
        WanDMAD(WanDMADConfig(net=cfg, teacher_ckpt=str(tmp_path / "bad.pth")), device="cpu", dtype=torch.float32)
