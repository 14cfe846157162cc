"""The EDM-stack FID tool against the reference's own fid.py pieces: the same image listing and subset
selection as its ImageFolderDataset, statistics equal to a direct float64 computation, and the same
Frechet distance as its calculate_fid_from_inception_stats; the CLI round trip (ref, then calc on the
same images) gives ~0."""
import os
import sys
import zipfile

import numpy as np
import pytest
import torch
from PIL import Image

from _reference_src import image_tree


class _Det(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.lin = torch.nn.Linear(3 * 16 * 16, 6)

    def forward(self, x, return_features: bool = True):
        return torch.tanh(self.lin(x.float().flatten(1) / 255.0))


@pytest.fixture()
def images(tmp_path):
    rng = np.random.RandomState(0)
    d = tmp_path / "imgs"
    (d / "sub").mkdir(parents=True)
    for i in range(11):
        arr = rng.randint(0, 256, (16, 16, 3), dtype=np.uint8)
        Image.fromarray(arr).save(d / ("sub" if i % 3 == 0 else "") / f"{i:03d}.png")
        grey = tmp_path / "grey"
        grey.mkdir(exist_ok=True)
        Image.fromarray(arr[:, :, 0]).save(grey / f"{i:03d}.png")
    (d / "notes.txt").write_text("not an image")
    z = tmp_path / "imgs.zip"
    with zipfile.ZipFile(z, "w") as zf:
        for root, _d, files in os.walk(d):
            for f in files:
                zf.write(os.path.join(root, f), os.path.relpath(os.path.join(root, f), d))
    torch.manual_seed(0)
    det = tmp_path / "det.pt"
    torch.jit.script(_Det()).save(str(det))
    return str(d), str(z), str(det)


def _reference_modules():
    edm = os.path.join(image_tree(), "third_party", "edm")
    if edm not in sys.path:
        sys.path.insert(0, edm)
    from training import dataset  # noqa: E402  (the reference's own module)
    import fid  # noqa: E402
    return dataset, fid


def test_listing_selection_and_stats_match_reference(images, monkeypatch):
    from dmad_b200.tools.edm_fid import ImageSource, inception_stats, load_detector, select_indices

    folder, zpath, det_path = images
    dataset, ref_fid = _reference_modules()
    det = load_detector(det_path, "cpu")
    for path in (folder, zpath):
        src = ImageSource(path)
        ref_ds = dataset.ImageFolderDataset(path=path, max_size=7, random_seed=3)
        assert src.names == ref_ds._image_fnames
        idx = select_indices(len(src), 7, 3)
        np.testing.assert_array_equal(idx, ref_ds._raw_idx)
        for k, i in enumerate(idx):
            np.testing.assert_array_equal(src.load(int(i)), ref_ds[k][0])
        mu, sigma = inception_stats(src, det, idx, batch=3)
        imgs = torch.from_numpy(np.stack([src.load(int(i)) for i in idx]))
        imgs = imgs.repeat(1, 3, 1, 1) if imgs.shape[1] == 1 else imgs
        f = det(imgs).detach().double().numpy()
        # float32 features in batches of 3 against one batch: rounding of the detector only
        np.testing.assert_allclose(mu, f.mean(0), rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(sigma, np.cov(f, rowvar=False), rtol=1e-5, atol=1e-7)
    # grey images enter the detector repeated to three channels
    grey = ImageSource(os.path.join(os.path.dirname(folder), "grey"))
    assert grey.load(0).shape == (1, 16, 16)
    mu_g, _ = inception_stats(grey, det, None, batch=4)
    rgb = torch.from_numpy(np.stack([grey.load(i) for i in range(len(grey))])).repeat(1, 3, 1, 1)
    np.testing.assert_allclose(mu_g, det(rgb).detach().double().numpy().mean(0), rtol=1e-5, atol=1e-7)
    from dmad_b200.samplers.edm import frechet_distance
    rng = np.random.RandomState(1)
    a, b = rng.randn(40, 6), rng.randn(50, 6) * 1.3 + 0.2
    m1, s1, m2, s2 = a.mean(0), np.cov(a, rowvar=False), b.mean(0), np.cov(b, rowvar=False)
    # the installed SciPy no longer takes sqrtm(..., disp=False), which the reference calls; restore the
    # old (result, error estimate) convention for the duration of the test
    import scipy.linalg
    plain = scipy.linalg.sqrtm
    monkeypatch.setattr(scipy.linalg, "sqrtm", lambda x, disp=True: (plain(x), 0.0) if not disp else plain(x))
    assert abs(frechet_distance(m1, s1, m2, s2) - ref_fid.calculate_fid_from_inception_stats(m1, s1, m2, s2)) < 1e-9


def test_cli_round_trip(images, tmp_path, capsys):
    from dmad_b200.tools.edm_fid import main

    folder, zpath, det_path = images
    dest = str(tmp_path / "refs" / "stats.npz")
    main(["ref", "--data", zpath, "--dest", dest, "--detector", det_path, "--device", "cpu", "--batch", "4"])
    ref = np.load(dest)
    assert ref["mu"].shape == (6,) and ref["sigma"].shape == (6, 6)
    fid = main(["calc", "--images", folder, "--ref", dest, "--num", "11", "--detector", det_path, "--device", "cpu"])
    assert abs(fid) < 1e-6
    with pytest.raises(SystemExit):
        main(["calc", "--images", folder, "--ref", dest, "--num", "50", "--detector", det_path, "--device", "cpu"])
