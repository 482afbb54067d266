"""B200-native (sm_100a) DeepSeek-V2 MoE block of the Unlimited-OCR decoder.

Import with ``importlib.import_module("unlimited-ocr-max_b200")`` (the directory name is
not a Python identifier). Public surface:

* ``MoEConfig``, ``UocrMoE`` -- the reference's ``MoE`` module surface (decoder.py:517-667);
* ``ops`` -- the reference's custom ops ``moe_bf16_qmv``, ``moe_int8_qmv``,
  ``int8_dequant_expert``, ``dense_bf16_qmv``, the gate ``route`` and the int8 quantiser
  ``quantize_per_group``;
* ``ep`` -- ``ExpertParallelMoE``, the prefill with routed experts sharded over GPUs;
* ``checkpoint`` -- safetensors reading and writing, ``load_moe_layer`` (one decoder layer's MoE
  from the model file) and ``quantize_checkpoint`` (the int8 checkpoint, quantised on the GPU);
* ``synth`` -- seeded synthetic weights and activations of the benchmark configs;
* ``build`` -- compiles ``libuocr_moe.so`` in-tree.
"""

from . import ops  # noqa: F401
from ._lib import LIB_PATH, load  # noqa: F401
from .moe import ConfigError, MoEConfig, UocrMoE  # noqa: F401
