"""Training entry points: bootstrap NTP, distributed bootstrap, GRPO, RL pretraining, flywheel, ACT-V."""
