"""Row-array LMDB datasets of the image stack with a dictionary-backed stand-in for the lmdb package
(the key layout of train/image/main/utils.py:56-77, create_lmdb_iterative.py), and the EDM
teacher-sample tool on a tiny network (seed + i per sample, label i mod label_dim)."""
import numpy as np
import torch


class _Txn:
    def __init__(self, store):
        self.store = store

    def get(self, k):
        return self.store.get(k)

    def put(self, k, v):
        self.store[k] = bytes(v)

    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


class _Env:
    def __init__(self):
        self.store = {}

    def begin(self, write=False):
        return _Txn(self.store)


def test_image_rows_roundtrip():
    from dmad_b200.data.lmdb_arrays import LMDBImageDataset, write_rows, write_shapes

    env = _Env()
    imgs = np.random.default_rng(0).integers(0, 256, size=(5, 3, 4, 4), dtype=np.uint8)
    labs = np.arange(5, dtype=np.int64) * 7
    write_rows(env, {"images": imgs[:3], "labels": labs[:3]}, 0)
    write_rows(env, {"images": imgs[3:], "labels": labs[3:]}, 3)
    write_shapes(env, {"images": imgs, "labels": labs}, 5)
    assert env.store[b"images_shape"] == b"5 3 4 4" and env.store[b"labels_shape"] == b"5"
    ds = LMDBImageDataset(env)
    assert len(ds) == 5
    item = ds[4]
    torch.testing.assert_close(item["images"], torch.tensor(imgs[4], dtype=torch.float32) / 255)
    assert int(item["class_labels"]) == 28


def test_latent_prompt_rows():
    from dmad_b200.data.lmdb_arrays import LMDBLatentPromptDataset, write_rows, write_shapes

    env = _Env()
    lat = np.random.default_rng(1).standard_normal((2, 4, 8, 8)).astype(np.float16)
    write_rows(env, {"latents": lat, "prompts": ["a cat", "a dog"]})
    write_shapes(env, {"latents": lat}, 2)

    class Tok:
        model_max_length = 6

        def __call__(self, texts, padding, max_length, truncation, return_tensors):
            ids = [[len(w) for w in texts[0].split()] + [0] * (max_length - len(texts[0].split()))]

            class R:
                input_ids = torch.tensor(ids)
            return R()

    ds = LMDBLatentPromptDataset(env, Tok())
    it = ds[1]
    assert it["prompt"] == "a dog" and it["text_input_ids_one"].shape == (1, 6)
    torch.testing.assert_close(it["images"], torch.tensor(lat[1].astype(np.float32)))


def test_edm_teacher_samples_tool():
    from dmad_b200.models.edm import EDMPrecond
    from dmad_b200.tools.edm_teacher_samples import generate, write_lmdb
    from dmad_b200.data.lmdb_arrays import LMDBImageDataset

    torch.manual_seed(0)
    net = EDMPrecond(8, 3, label_dim=10, model_channels=16, channel_mult=(1,), num_blocks=1, attn_resolutions=()).eval()
    imgs, labs = generate(net, [0, 1, 2, 13], seed=10, label_dim=10, steps=3, batch=3)
    assert imgs.dtype == np.uint8 and imgs.shape == (4, 3, 8, 8) and labs.tolist() == [0, 1, 2, 3]
    again, _ = generate(net, [13], seed=10, label_dim=10, steps=3, batch=1)
    assert np.array_equal(again[0], imgs[3])  # per-sample seeds: independent of the batching
    env = _Env()
    write_lmdb(env, imgs, labs, 0, 4)
    assert len(LMDBImageDataset(env)) == 4
