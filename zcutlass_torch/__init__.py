"""The reference's import name `zcutlass_torch`, served by zcutlass_b200.zcutlass_torch.

`import zcutlass_torch` and `import zcutlass_torch.overlay` give the
implementation package and its module themselves (one module object each,
so overlay state and isinstance checks are shared with zcutlass_b200)."""

import sys

from zcutlass_b200 import zcutlass_torch as _impl
from zcutlass_b200.zcutlass_torch import overlay as _overlay

sys.modules[__name__ + ".overlay"] = _overlay
sys.modules[__name__] = _impl
