"""saint_llm_b200 -- a Blackwell-native (sm_100a) DeepSeek-V4-style training and
inference framework with the capabilities of iZonex/saint-llm."""

from saint_llm_b200.config import ModelConfig, RunConfig

__version__ = "0.1.0"

__all__ = ["ModelConfig", "RunConfig", "__version__"]
