"""``python -m dmad_b200.cli.train --config configs/wan_1p3b_dmad.yaml [--dryrun] [key.sub=value ...]``

One process per GPU (launch with ``torchrun --nproc-per-node N``).  Parity: the Wan entry
(train/wan/scripts/train.py:107-160: config + overrides, ``--dryrun``, distributed init, trainer)
and the H3 entry (train/h3/train.py:11-34: ``--config``, TF32, init, train, cleanup).
"""
from __future__ import annotations

import argparse
import sys

import torch


def main(argv=None):
    ap = argparse.ArgumentParser(description="DMAD / rCM distillation training")
    ap.add_argument("--config", default=None, help="YAML config (see configs/)")
    ap.add_argument("--dryrun", action="store_true", help="build everything, run one iteration, exit")
    ap.add_argument("--print-config", action="store_true", help="print the resolved config and exit")
    ap.add_argument("overrides", nargs="*", help="key.sub=value overrides; experiment=<name> selects a preset")
    a = ap.parse_args(argv)
    from ..runtime.config import load_config
    from . import presets  # noqa: F401  (registers the named experiments)

    cfg = load_config(a.config, a.overrides)
    if a.print_config:
        import yaml
        yaml.safe_dump(cfg, sys.stdout, sort_keys=False)
        return 0
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.backends.cudnn.allow_tf32 = True
    from ..train.trainer import DistillTrainer

    tr = DistillTrainer(cfg, dryrun=a.dryrun)
    try:
        tr.train()
    finally:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
