"""Import path of the reference's zcutlass_vllm.plugin module."""

from zcutlass_b200.zcutlass_vllm.plugin import *  # noqa: F401,F403
