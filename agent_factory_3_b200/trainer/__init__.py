"""Training side: ModelTrainer (packed LoRA / full-parameter steps on gpt-oss), the async RL
loop (RLFlow), sample processing, weight sync to the rollout engines, checkpoints and the
rollout saver / reader."""
