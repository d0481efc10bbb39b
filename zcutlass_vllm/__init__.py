"""Import name of the reference's vLLM package; the implementation lives in
zcutlass_b200.zcutlass_vllm."""

from zcutlass_b200.zcutlass_vllm import *  # noqa: F401,F403
from zcutlass_b200.zcutlass_vllm import __all__  # noqa: F401
