"""GRINQH quantized linear for vLLM, sm_100a (B200) kernels.

``register`` is the ``vllm.general_plugins`` entry point (same as the reference's
``grinqh/__init__.py:1-2``); vLLM calls it in every process, and importing the
module twice is harmless.
"""


def register():
    from . import grinqh  # noqa: F401  (runs @register_quantization_config)
