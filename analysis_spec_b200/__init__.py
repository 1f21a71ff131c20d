"""B200 (sm_100a) static-KV-cache and tree-verify path for tree speculative decoding.

Drop-in modules mirroring the reference's ``helper`` package:
  opd_static_cache   OPDStaticCache / StaticAppendLayer / swap_remove_plan / persistent_cache
  opd_kv_kernels     remap_rows / move_tail_rows
  opd_scheduling     schedule / compact_suffix_inplace
  tree_kernels       kernel plugin (tree_mask, trace_path, pad_verified_path, pad_schedule)
  tree_verification  PackedTree / pack_tree / VerifiedPath / trace_verified_path
  tree_attention     AttentionInterface function for the verify forward
All compute runs in libspeckv.so (hand-written sm_100a CUDA, C ABI in include/speckv.h).
"""
__version__ = '0.1.0'
