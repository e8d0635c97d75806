"""Shapes for add_rmsnorm_fp8_quant (default = BASELINE second config)."""
SINGLE_SHAPES = {"default": {"shape": [8192, 8192], "eps": 1e-6, "dtype": "BF16"}}
SHAPE_FAMILIES = {
    "shape_sweep": [
        {"shape": [1, 4096], "eps": 1e-6, "dtype": "BF16"},
        {"shape": [64, 8192], "eps": 1e-6, "dtype": "BF16"},
        {"shape": [2048, 4096], "eps": 1e-6, "dtype": "BF16"},
        {"shape": [8192, 8192], "eps": 1e-6, "dtype": "BF16"},
        {"shape": [4, 512, 4096], "eps": 1e-6, "dtype": "BF16"},
    ],
    "dtype_sweep": [
        {"shape": [512, 4096], "eps": 1e-6, "dtype": "FP32"},
        {"shape": [512, 4096], "eps": 1e-6, "dtype": "FP16"},
        {"shape": [512, 4096], "eps": 1e-6, "dtype": "BF16"},
    ],
}
RANDOM_SHAPE_SPACE = {"shape": [[1, 4096], [128, 4096], [2048, 8192], [8192, 8192], [16, 1, 8192]],
                      "eps": [1e-6, 1e-5], "dtype": ["FP32", "FP16", "BF16"]}
