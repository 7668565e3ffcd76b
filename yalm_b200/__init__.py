"""yalm_b200 — B200-native batch-1 decode engine for yalm .yalm checkpoints.

The product is the native library libyalm_b200.so (C ABI: include/yalm_b200.h).  This package is
its host-side mirror of yalm's model interface (model.py), the .yalm reader (codec.py), the
synthetic checkpoint writer (synth.py) and the build script (build.py).
"""
from ._lib import YalmB200Error, MODE_HYDRATE, MODE_LOGITS  # noqa: F401
from .codec import YALMData  # noqa: F401
from .model import Config, InferenceMode, InferenceState, Model, positions  # noqa: F401
