"""Import path of the reference's zcutlass_vllm.linear_method module."""

from zcutlass_b200.zcutlass_vllm.linear_method import *  # noqa: F401,F403
