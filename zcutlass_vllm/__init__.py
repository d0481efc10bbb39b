"""The reference's import name `zcutlass_vllm`, served by zcutlass_b200.zcutlass_vllm.

`import zcutlass_vllm` and `import zcutlass_vllm.<module>` (linear,
linear_method, oot_linear, plugin, route_logger -- the names vLLM's plugin
entry point and the reference's tools import) give the implementation
package and its modules themselves, one module object each."""

import importlib
import sys

from zcutlass_b200 import zcutlass_vllm as _impl

for _name in ("linear", "linear_method", "oot_linear", "plugin", "route_logger"):
    sys.modules[f"{__name__}.{_name}"] = importlib.import_module(f"zcutlass_b200.zcutlass_vllm.{_name}")
sys.modules[__name__] = _impl
