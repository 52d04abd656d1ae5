"""Which modules of an OLMo model are quantised, in execution order.  The reference declares this for AutoGPTQ in a class of
this module (``OLMoGPTQForCausalLM``: block container, modules outside the blocks, linears inside a block); the quantiser
of this framework (:mod:`olmo_b200.inference.quantize`) reads the same three facts from here."""
from olmo_b200.inference.quantize import BLOCK_LINEARS


class OLMoGPTQForCausalLM:
    """Layout description; not a model class (quantise with ``olmo_b200.inference.quantize.quantize_model``)."""

    layers_block_name = "transformer.blocks"
    outside_layer_modules = ["transformer.wte", "transformer.ln_f"]
    inside_layer_modules = [[name] for name in BLOCK_LINEARS]


__all__ = ["OLMoGPTQForCausalLM"]
