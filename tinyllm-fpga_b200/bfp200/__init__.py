"""bfp200 -- B200-native block-floating-point SmolLM2-135M greedy decode.

A drop-in replacement for the bit-exact BFP simulator of jrrk2/tinyllm-fpga
(rtl/vc707/host/gen_smollm_blockfp_full.py): the same packed image / ROM
files in, the same greedy token stream out, computed by hand-written sm_100a
kernels behind the C ABI of include/bfp200.h (libbfp200.so, built in-tree by
``bfp200.build``).

Modules
-------
config   BfpConfig (reference env-var names)
image    DDR3 region map, .hex ROM files, cfg.svh, token files
pack     quantize_W (GPU), byte-exact DDR3 image packing
synth    seeded synthetic model + benchmark prompts
ops      op-level GPU functions (tile_quantize, matvec, rmsnorm_fp, ...)
engine   Decoder (one GPU), generate_multi (sequence-parallel, no collectives),
         shard_group / generate_sharded (vocabulary-sharded head, NCCL)
dist     one process per GPU: step-balanced sequence partition, token gather,
         sharded-head argmax exchange (torch.distributed)
sim      drop-in facade with the reference module's names
"""
from ._lib import BfpError
from .config import BfpConfig, SMOLLM2_135M
from .engine import Decoder, generate_multi, generate_sharded, nccl_unique_id, shard_group

__all__ = ["BfpError", "BfpConfig", "SMOLLM2_135M", "Decoder", "generate_multi", "generate_sharded",
           "nccl_unique_id", "shard_group"]
