"""Training-session API shared by ``train_zero.py`` and ``bench.py``."""

from .session import SessionConfig, TrainSession, broadcast_model, init_distributed, model_param_dtype

__all__ = ["SessionConfig", "TrainSession", "broadcast_model", "init_distributed", "model_param_dtype"]
