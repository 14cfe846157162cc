"""Row-array LMDB datasets of the image stack (EDM ImageNet images, SDXL latents + prompts, teacher samples).

Parity: train/image/main/data/lmdb_dataset.py:12-53 (``LMDBDataset``: uint8 images / 255 and int64
labels), train/image/main/sd_image_dataset.py:7-60 (``SDImageDatasetLMDB``: fp16 latents and prompts,
tokenised per item), train/image/main/data/create_lmdb_iterative.py:9-79 (the writer) and the row
helpers of train/image/main/utils.py:56-77.  Layout, kept so existing databases open: key
``<name>_<i>_data`` holds the raw bytes of row ``i`` of array ``name`` (UTF-8 for strings) and key
``<name>_shape`` the ASCII shape ``"N d1 d2 ..."`` of the whole array.

The ``lmdb`` package is optional: ``open_env`` imports it on first use and says how to get it when it
is missing.  Any object with ``begin(write=False)`` returning a transaction with ``get`` / ``put``
(and context-manager support) works as the environment, which is how the tests run without it.
"""
from __future__ import annotations

import numpy as np
import torch
from torch.utils.data import Dataset


def open_env(path: str, readonly: bool = True, map_size: int = 1 << 40):
    try:
        import lmdb
    except ImportError as exc:  # pragma: no cover - depends on the environment
        raise ImportError("reading or writing LMDB datasets needs the `lmdb` package "
                          "(pip install lmdb); the tar-shard format (dmad_b200.data.shards) needs nothing") from exc
    if readonly:
        return lmdb.open(path, readonly=True, lock=False, readahead=False, meminit=False)
    return lmdb.open(path, map_size=map_size)


def array_shape(env, name: str) -> tuple:
    with env.begin() as txn:
        raw = txn.get(f"{name}_shape".encode())
    if raw is None:
        raise KeyError(f"array {name!r} has no shape record")
    return tuple(int(x) for x in bytes(raw).decode().split())


def read_row(env, name: str, dtype, shape, index: int):
    with env.begin() as txn:
        raw = txn.get(f"{name}_{index}_data".encode())
    if raw is None:
        raise IndexError(f"{name}[{index}] is not in the database")
    a = np.frombuffer(bytes(raw), dtype=dtype)
    return a.reshape(shape) if len(shape) else a


def read_string(env, name: str, index: int) -> str:
    with env.begin() as txn:
        raw = txn.get(f"{name}_{index}_data".encode())
    if raw is None:
        raise IndexError(f"{name}[{index}] is not in the database")
    return bytes(raw).decode()


def write_rows(env, arrays: dict, start_index: int = 0) -> int:
    """Stores every row of every array (numpy arrays, tensors or lists of strings) from ``start_index``;
    returns the number of rows written per array."""
    n = None
    with env.begin(write=True) as txn:
        for name, arr in arrays.items():
            if torch.is_tensor(arr):
                arr = arr.cpu().numpy()
            for i, row in enumerate(arr):
                data = row.encode() if isinstance(row, str) else np.ascontiguousarray(row).tobytes()
                txn.put(f"{name}_{start_index + i}_data".encode(), data)
            n = len(arr) if n is None else n
    return n or 0


def write_shapes(env, arrays: dict, total_rows: int):
    """The ``<name>_shape`` records: the row shape of each array with the first dimension ``total_rows``."""
    with env.begin(write=True) as txn:
        for name, arr in arrays.items():
            shape = [total_rows] + (list(arr.shape[1:]) if hasattr(arr, "shape") else [])
            txn.put(f"{name}_shape".encode(), " ".join(str(int(x)) for x in shape).encode())


class LMDBImageDataset(Dataset):
    """``{"images": float [C, H, W] in [0, 1], "class_labels": long}`` per row (EDM / ImageNet)."""

    def __init__(self, path_or_env):
        self.env = open_env(path_or_env) if isinstance(path_or_env, str) else path_or_env
        self.image_shape = array_shape(self.env, "images")
        self.label_shape = array_shape(self.env, "labels")

    def __len__(self):
        return self.image_shape[0]

    def __getitem__(self, idx):
        img = read_row(self.env, "images", np.uint8, self.image_shape[1:], idx)
        lab = read_row(self.env, "labels", np.int64, self.label_shape[1:], idx)
        return {"images": torch.tensor(img, dtype=torch.float32) / 255.0,
                "class_labels": torch.tensor(lab, dtype=torch.long)}


class LMDBLatentPromptDataset(Dataset):
    """``{"images": float latents, "prompt": str}`` per row (SDXL); with tokenizers (Hugging Face
    callables) also ``text_input_ids_one`` / ``text_input_ids_two`` padded to their maximum length."""

    def __init__(self, path_or_env, tokenizer_one=None, tokenizer_two=None):
        self.env = open_env(path_or_env) if isinstance(path_or_env, str) else path_or_env
        self.latent_shape = array_shape(self.env, "latents")
        self.tok1, self.tok2 = tokenizer_one, tokenizer_two

    def __len__(self):
        return self.latent_shape[0]

    def _ids(self, tok, prompt):
        return tok([prompt], padding="max_length", max_length=tok.model_max_length, truncation=True,
                   return_tensors="pt").input_ids

    def __getitem__(self, idx):
        lat = read_row(self.env, "latents", np.float16, self.latent_shape[1:], idx)
        prompt = read_string(self.env, "prompts", idx)
        out = {"images": torch.tensor(lat.astype(np.float32)), "prompt": prompt}
        if self.tok1 is not None:
            out["text_input_ids_one"] = self._ids(self.tok1, prompt)
        if self.tok2 is not None:
            out["text_input_ids_two"] = self._ids(self.tok2, prompt)
        return out
