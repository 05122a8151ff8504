"""Full-MAML callers of the SDPA operator (``theria.maml``), plus the
BASELINE sequence-classification model and task sampler and the
task-sharded multi-GPU meta-step."""
