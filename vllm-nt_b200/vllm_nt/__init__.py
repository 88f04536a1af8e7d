"""vllm_nt -- vLLM general plugin whose hooked decoder ops run on hand-written sm_100a
kernels.  vLLM loads it through the ``vllm.general_plugins`` entry point
``vllm_nt = "vllm_nt:register"``; ``register`` imports ``vllm_nt.oot``, which applies the
hooks once per process."""

import os

if os.environ.get("VLLM_NT_ENABLE_CUSTOM_OP_REGISTER_INTERCEPT") == "1":
    __import__("vllm_nt.oot")


def register() -> None:
    __import__("vllm_nt.oot")
