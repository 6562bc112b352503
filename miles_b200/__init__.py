"""miles_b200: a Blackwell-native (sm_100a) RL post-training framework.

Trainer and rollout engine are both owned by this package; their hot ops are hand-written
sm_100a CUDA kernels (miles_b200/csrc) exposed through miles_b200.ops.
"""
__version__ = "0.1.0"
