"""Named experiments (``experiment=<name>`` on the command line).

Parity: the DMAD / rCM experiment configs of the Wan stack
(train/wan/rcm/configs/experiments/dmad/wan2pt1_t2v.py:33-101: 1.3B on 8 GPUs with batch 8,
``student_update_freq=2``, lr 2e-6, betas (0, 0.99); 14B on CP 8 with lr 1e-6) and the rCM
experiments (experiments/rcm/wan2pt1_t2v.py, sCM loss on).
"""
from ..runtime.config import experiment, merge, register_experiment

_COMMON = {"data": {"kind": "synthetic", "batch_size": 1, "latent_shape": [16, 21, 60, 104],
                    "text_shape": [512, 4096]},
           "training": {"max_iters": 10000, "save_every": 500, "save_total_limit": 3, "log_every": 10,
                        "auto_resume": True, "timeout_s": 3600, "heartbeat_s": 30,
                        "lr_schedule": "lambda_linear"}}  # the Wan stack's default scheduler

register_experiment("dmad_wan2pt1_1pt3b", {
    **_COMMON,
    "model": {"family": "wan_dmad", "net": "wan2.1-1.3b",
              "distill": {"lr": 2e-6, "critic_lr": 2e-6, "betas": [0.0, 0.99], "student_update_freq": 2,
                          "p_D_shift": 5.0, "checkpoint_critic_blocks_student_phase": 30}},
    "parallel": {"cp": 1, "dp_optimizer": "sharded"},
})

register_experiment("dmad_wan2pt1_14b_cp8", {
    **_COMMON,
    "model": {"family": "wan_dmad", "net": "wan2.1-14b",
              "distill": {"lr": 1e-6, "critic_lr": 1e-6, "betas": [0.0, 0.99], "student_update_freq": 2,
                          "student_lora_rank": 128, "checkpoint_student_blocks": 40, "shard_frozen": True,
                          "checkpoint_student_policy": "mm_only",
                          "checkpoint_critic_blocks": 40, "checkpoint_critic_blocks_student_phase": 40}},
    "parallel": {"cp": 8, "cp_impl": "fused", "dp_optimizer": "sharded"},
})

register_experiment("rcm_wan2pt1_1pt3b", {
    **_COMMON,
    "model": {"family": "wan_dmad", "net": "wan2.1-1.3b",
              "distill": {"loss_scale": 100.0, "cm_type": "scm", "critic_mode": "dmd", "tangent_warmup": 1000,
                          "lr": 2e-6, "critic_lr": 2e-6}},
    "parallel": {"cp": 1, "dp_optimizer": "sharded"},
})


# ``<name>_debug`` twins of every experiment: 25 iterations, log every 2, checkpoint every 10, no resume,
# tangent warm-up 8 (experiments/rcm/wan2pt1_t2v.py:23-58, registered for every job at :234)
_DEBUG = {"training": {"max_iters": 25, "log_every": 2, "save_every": 10, "auto_resume": False},
          "model": {"distill": {"tangent_warmup": 8}}}
for _name in ("dmad_wan2pt1_1pt3b", "dmad_wan2pt1_14b_cp8", "rcm_wan2pt1_1pt3b"):
    register_experiment(_name + "_debug", merge(experiment(_name), _DEBUG))
