"""Training-session API shared by ``train_zero.py`` and ``bench.py``."""

from .session import AsyncLoss, SessionConfig, TrainSession, broadcast_model, init_distributed, model_param_dtype

__all__ = ["AsyncLoss", "SessionConfig", "TrainSession", "broadcast_model", "init_distributed", "model_param_dtype"]
