"""Hot ops of brain_b200: thin autograd front-ends over the sm_100a kernels in ``csrc/``.

CUDA tensors always run the native kernels (an unbuilt library raises ``NativeMissing``);
CPU tensors run a float32 PyTorch restatement of the same op, which is also the test oracle.
"""
from . import _common  # noqa: F401  (registers signatures)
from ._common import check_status  # noqa: F401
from .gemm import gemm  # noqa: F401
from .norms import rms_norm, layer_norm, add_rms_norm, add_layer_norm, fused_layer_norm  # noqa: F401
from .activations import swiglu, gelu  # noqa: F401
from .rope import rope_table, apply_rope, apply_rope_  # noqa: F401
from .attention import flash_attention, flash_attention_fwd, qkv_attention, sdpa_ref  # noqa: F401
from .linear import linear, norm_linear, swiglu_linear, gelu_mlp  # noqa: F401
from .cross_entropy import cross_entropy, linear_cross_entropy  # noqa: F401
from .embedding import embedding  # noqa: F401
from .decode import paged_decode_attention, kv_append_rope  # noqa: F401
from . import optim_kernels  # noqa: F401
