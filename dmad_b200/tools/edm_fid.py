"""FID of generated images against dataset statistics, as the EDM image stack measures it.

Counterpart of the reference's ``train/image/third_party/edm/fid.py`` (``calc`` :112-137 and ``ref``
:141-160): the same two commands and flags, the same image listing (every file under a folder or in a zip
whose extension PIL reads, sorted by relative name; grey images repeated to three channels, uint8 NCHW into
the detector), the same subset for ``--num`` / ``--seed`` (a ``RandomState(seed)`` shuffle of the indices,
the first ``num`` kept in index order), float64 statistics accumulated as sums of features and outer
products (unbiased covariance) and the same Frechet distance.

The detector is the caller's Inception-v3 feature network, as in the reference (which downloads NVIDIA's
``inception-2015-12-05.pkl``): a TorchScript file is loaded with ``torch.jit.load``; the reference's
pickle itself is read only with ``--trust-pickle`` (unpickling runs code from the file).  It is called as
``detector(images, return_features=True)`` and returns [N, F] features.

    python -m dmad_b200.tools.edm_fid ref --data datasets/imagenet-64x64.zip --dest fid-refs/imagenet-64x64.npz \\
        --detector inception-2015-12-05.pt
    python -m dmad_b200.tools.edm_fid calc --images samples/ --ref fid-refs/imagenet-64x64.npz \\
        --detector inception-2015-12-05.pt
"""
from __future__ import annotations

import argparse
import os
import pickle
import zipfile

import numpy as np
import torch
from PIL import Image

from ..samplers.edm import frechet_distance


class ImageSource:
    """The image files of a folder (recursively) or a zip archive, in sorted relative-name order."""

    def __init__(self, path: str):
        self.path = path
        self._zip = None
        if os.path.isdir(path):
            names = {os.path.relpath(os.path.join(root, f), start=path) for root, _d, files in os.walk(path)
                     for f in files}
        elif os.path.splitext(path)[1].lower() == ".zip":
            self._zip = zipfile.ZipFile(path)
            names = set(self._zip.namelist())
        else:
            raise OSError(f"{path}: need a folder or a .zip of images")
        Image.init()
        self.names = sorted(n for n in names if os.path.splitext(n)[1].lower() in Image.EXTENSION)
        if not self.names:
            raise OSError(f"{path}: no image files")

    def __len__(self):
        return len(self.names)

    def load(self, i: int) -> np.ndarray:
        """uint8 CHW (grey images as one channel)."""
        name = self.names[i]
        if self._zip is not None:
            with self._zip.open(name, "r") as f:
                img = np.array(Image.open(f))
        else:
            with open(os.path.join(self.path, name), "rb") as f:
                img = np.array(Image.open(f))
        if img.ndim == 2:
            img = img[:, :, None]
        return img.transpose(2, 0, 1)


def select_indices(n: int, num: int | None, seed: int = 0) -> np.ndarray:
    """Indices of the images used: all of them, or ``num`` chosen by a seeded shuffle, in index order."""
    idx = np.arange(n, dtype=np.int64)
    if num is not None and n > num:
        np.random.RandomState(seed % (1 << 31)).shuffle(idx)
        idx = np.sort(idx[:num])
    return idx


def load_detector(path: str, device, trust_pickle: bool = False):
    try:
        net = torch.jit.load(path, map_location=device)
    except (RuntimeError, ValueError) as e:
        if not trust_pickle:
            raise ValueError(f"{path} is not a TorchScript file; pass --trust-pickle to unpickle it (this runs "
                             f"code from the file, as the reference does)") from e
        with open(path, "rb") as f:
            net = pickle.load(f)  # noqa: S301 - explicitly requested by the caller
        net = net.to(device)
    return net.eval()


@torch.no_grad()
def batch_stats(batches, detector, device="cpu"):
    """(mu, sigma) in float64 of the detector's features over uint8 NCHW image batches."""
    mu = sigma = None
    n = 0
    for imgs in batches:
        if imgs.shape[1] == 1:
            imgs = imgs.repeat(1, 3, 1, 1)
        try:
            f = detector(imgs.to(device), return_features=True)
        except TypeError:
            f = detector(imgs.to(device))
        f = f.to(torch.float64)
        if mu is None:
            mu = torch.zeros(f.shape[1], dtype=torch.float64, device=f.device)
            sigma = torch.zeros(f.shape[1], f.shape[1], dtype=torch.float64, device=f.device)
        mu += f.sum(0)
        sigma += f.T @ f
        n += f.shape[0]
    if n < 2:
        raise ValueError(f"need at least 2 images to compute statistics, found {n}")
    mu /= n
    sigma -= torch.outer(mu, mu) * n
    sigma /= n - 1
    return mu.cpu().numpy(), sigma.cpu().numpy()


def inception_stats(source: ImageSource, detector, indices=None, batch: int = 64, device="cpu"):
    """(mu, sigma) in float64 of the detector's features over the selected images."""
    idx = np.arange(len(source)) if indices is None else np.asarray(indices)
    if len(idx) < 2:
        raise ValueError(f"need at least 2 images to compute statistics, found {len(idx)}")
    batches = (torch.from_numpy(np.stack([source.load(int(i)) for i in idx[s:s + batch]]))
               for s in range(0, len(idx), batch))
    return batch_stats(batches, detector, device)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("calc", help="FID of a set of images against reference statistics")
    c.add_argument("--images", required=True, help="folder or zip of images")
    c.add_argument("--ref", required=True, help="npz with mu / sigma")
    c.add_argument("--num", type=int, default=50000, help="number of images to use")
    c.add_argument("--seed", type=int, default=0, help="seed of the image selection")
    c.add_argument("--batch", type=int, default=64)
    r = sub.add_parser("ref", help="reference statistics of a dataset")
    r.add_argument("--data", required=True, help="folder or zip of images")
    r.add_argument("--dest", required=True, help="destination .npz")
    r.add_argument("--batch", type=int, default=64)
    for p in (c, r):
        p.add_argument("--detector", required=True, help="Inception-v3 feature network (TorchScript, or the "
                                                         "reference's pickle with --trust-pickle)")
        p.add_argument("--trust-pickle", action="store_true")
        p.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    det = load_detector(a.detector, a.device, a.trust_pickle)
    if a.cmd == "calc":
        ref = dict(np.load(a.ref))
        src = ImageSource(a.images)
        if len(src) < a.num:
            raise SystemExit(f"found {len(src)} images, but expected at least {a.num}")
        mu, sigma = inception_stats(src, det, select_indices(len(src), a.num, a.seed), a.batch, a.device)
        fid = frechet_distance(mu, sigma, ref["mu"], ref["sigma"])
        print(f"{fid:g}")
        return fid
    src = ImageSource(a.data)
    mu, sigma = inception_stats(src, det, None, a.batch, a.device)
    if os.path.dirname(a.dest):
        os.makedirs(os.path.dirname(a.dest), exist_ok=True)
    np.savez(a.dest, mu=mu, sigma=sigma)
    print(f"saved {a.dest}")
    return None


if __name__ == "__main__":
    main()
