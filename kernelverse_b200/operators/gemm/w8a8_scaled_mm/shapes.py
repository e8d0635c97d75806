"""Shapes for w8a8_scaled_mm (default = BASELINE third config, M = 256)."""
SINGLE_SHAPES = {"default": {"M": 256, "N": 28672, "K": 8192}}
SHAPE_FAMILIES = {
    "shape_sweep": [
        {"M": 16, "N": 28672, "K": 8192},
        {"M": 256, "N": 28672, "K": 8192},
        {"M": 4096, "N": 28672, "K": 8192},
    ],
}
RANDOM_SHAPE_SPACE = {"M": [1, 16, 128, 256, 1024, 4096], "N": [1024, 4096, 11008, 28672], "K": [1024, 4096, 8192]}
