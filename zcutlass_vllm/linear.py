"""Import path of the reference's zcutlass_vllm.linear module."""

from zcutlass_b200.zcutlass_vllm.linear import *  # noqa: F401,F403
