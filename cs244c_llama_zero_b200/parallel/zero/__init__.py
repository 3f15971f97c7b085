"""ZeRO engines, stages 0-3 (reference ``zero/``)."""

from .stage012 import ZeROStage0DDP, ZeROStage1Optimizer, ZeROStage2Optimizer
from .stage3 import ZeROStage3Optimizer

ENGINES = {0: ZeROStage0DDP, 1: ZeROStage1Optimizer, 2: ZeROStage2Optimizer, 3: ZeROStage3Optimizer}

__all__ = ["ZeROStage0DDP", "ZeROStage1Optimizer", "ZeROStage2Optimizer", "ZeROStage3Optimizer", "ENGINES"]
