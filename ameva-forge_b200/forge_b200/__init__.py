"""forge_b200: the B200-native quantized-LLM inference path of AMEVA-Forge.

Host-side mirror of the reference's op API (gpuCore) and model API
(LlamaForCausalLM) over libforge_b200.so, the sm_100a CUDA library whose C
ABI is include/forge_b200.h.
"""
from . import errors
from ._capi import LIB_PATH, lib
from .gpu_core import Context, default, device_count, init, nccl_unique_id
from .gguf import GGUFFile
from .graph import GraphBuilder, configure_graph, execute_graph
from .llama import LLAMA2_7B, TINYLLAMA_1_1B, LlamaConfig, LlamaForCausalLM

__all__ = ["GraphBuilder", "configure_graph", "execute_graph", "errors", "LIB_PATH", "lib", "Context", "default", "device_count", "init", "nccl_unique_id",
           "GGUFFile", "LlamaConfig", "LlamaForCausalLM", "LLAMA2_7B", "TINYLLAMA_1_1B"]
