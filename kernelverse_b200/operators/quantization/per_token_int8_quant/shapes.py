"""Shapes for per_token_int8_quant (default = BASELINE first config)."""
SINGLE_SHAPES = {"default": {"num_tokens": 2048, "hidden_dim": 4096, "dtype": "BF16"}}
SHAPE_FAMILIES = {
    "shape_sweep": [
        {"num_tokens": 1, "hidden_dim": 4096, "dtype": "BF16"},
        {"num_tokens": 16, "hidden_dim": 4096, "dtype": "BF16"},
        {"num_tokens": 2048, "hidden_dim": 4096, "dtype": "BF16"},
        {"num_tokens": 8192, "hidden_dim": 8192, "dtype": "BF16"},
    ],
    "dtype_sweep": [
        {"num_tokens": 2048, "hidden_dim": 4096, "dtype": "FP32"},
        {"num_tokens": 2048, "hidden_dim": 4096, "dtype": "FP16"},
        {"num_tokens": 2048, "hidden_dim": 4096, "dtype": "BF16"},
    ],
}
RANDOM_SHAPE_SPACE = {"num_tokens": [1, 16, 128, 2048, 8192], "hidden_dim": [1024, 4096, 8192, 11008],
                      "dtype": ["FP32", "FP16", "BF16"]}
