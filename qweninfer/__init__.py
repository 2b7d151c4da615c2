"""QwenInfer's public import path (`qweninfer.models.qwen2`, `qweninfer.engine.engine`, ...)
over the B200 implementation in `qweninfer_b200`.

Code written against QwenInfer keeps its imports; every module here re-exports the
names of the QwenInfer module of the same path (qweninfer/models/{config,qwen2}.py,
qweninfer/engine/{kv_cache,engine,generate}.py) from its qweninfer_b200 counterpart.
The benchmark harnesses of `qweninfer.bench` are not part of this package.
"""

__version__ = "0.1.0"
