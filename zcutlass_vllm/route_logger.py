"""Import path of the reference's zcutlass_vllm.route_logger module."""

from zcutlass_b200.zcutlass_vllm.route_logger import *  # noqa: F401,F403
