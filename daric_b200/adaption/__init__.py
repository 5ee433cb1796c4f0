"""Re-rotation and recompute policy (drop-in for ``daric.adaption``)."""
from .adapter import Adapter, AdaptionConfig
from .policy import DARICPolicy, cluster_groups

__all__ = ["Adapter", "AdaptionConfig", "DARICPolicy", "cluster_groups"]
