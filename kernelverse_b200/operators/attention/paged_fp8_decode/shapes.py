"""Shapes for paged_fp8_decode (default = BASELINE fourth config)."""
_BASE = {"batch_size": 64, "num_q_heads": 32, "num_kv_heads": 8, "head_dim": 128, "block_size": 16,
         "min_context": 512, "max_context": 8192}
SINGLE_SHAPES = {"default": dict(_BASE)}
SHAPE_FAMILIES = {
    "shape_sweep": [
        dict(_BASE, batch_size=4, min_context=16, max_context=512),
        dict(_BASE, batch_size=16, min_context=512, max_context=4096),
        dict(_BASE),
        dict(_BASE, num_q_heads=8, num_kv_heads=1),
        dict(_BASE, head_dim=64),
    ],
}
RANDOM_SHAPE_SPACE = {"batch_size": [1, 8, 64], "num_q_heads": [8, 32], "num_kv_heads": [1, 8], "head_dim": [64, 128],
                      "block_size": [8, 16, 32], "min_context": [1, 512], "max_context": [1024, 8192]}
