"""B200-native Q4 decode backend for MicroLLM lab (hand-written sm_100a CUDA behind a C ABI).

Import with ``importlib.import_module("microllm-lab_b200")`` (the directory name holds a hyphen).
"""
from .engine import (CudaPetitGPT, DTYPES, MllmError, SPECIAL, gemm_q4_device, gemv_device, gemv_q4_device, load_library,
                     LIB_PATH, EXPORTS)
from .pgw import (CONFIGS, Bundle, copy_span_prompt, dequant_q4, parse_pgw, quant_q4, quant_q8, seeded_prompt,
                  synthetic_pgw, write_pgw)
from .tokenizer import Tokenizer, encode_messages
from .worker import DecodeWorker

__all__ = ["CudaPetitGPT", "DTYPES", "MllmError", "SPECIAL", "gemm_q4_device", "gemv_device", "gemv_q4_device", "load_library", "LIB_PATH", "EXPORTS", "CONFIGS",
           "Bundle", "copy_span_prompt", "dequant_q4", "parse_pgw", "quant_q4", "quant_q8", "seeded_prompt", "synthetic_pgw",
           "write_pgw", "DecodeWorker", "Tokenizer", "encode_messages"]
