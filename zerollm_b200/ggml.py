"""ggml tensor types and row sizes (src/gguf/types.js:10-65, src/compute/ref-kernels.js:65-77)."""
F32, F16, Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 2, 6, 8, 12, 13, 14, 30

# type id -> (name, values per block, bytes per block)  (types.js:24-54)
TYPE_INFO = {
    F32: ("F32", 1, 4), F16: ("F16", 1, 2), BF16: ("BF16", 1, 2),
    Q4_0: ("Q4_0", 32, 18), Q5_0: ("Q5_0", 32, 22), Q8_0: ("Q8_0", 32, 34),
    Q4_K: ("Q4_K", 256, 144), Q5_K: ("Q5_K", 256, 176), Q6_K: ("Q6_K", 256, 210),
}
NAMES = {v[0]: k for k, v in TYPE_INFO.items()}

# config.js:12-15
SUPPORTED_TENSOR_TYPES = frozenset(TYPE_INFO)
QUANTIZED = frozenset({Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K})


def type_name(t: int) -> str:
    return TYPE_INFO[t][0] if t in TYPE_INFO else f"type{t}"


def row_bytes(t: int, cols: int) -> int:
    """Bytes in one row of ``cols`` values (types.js:60-65): raises like rowSize."""
    if t not in TYPE_INFO:
        raise ValueError(f"reference kernels: unsupported tensor type {t} (supported: F32, F16, BF16, Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K)")
    name, bs, ts = TYPE_INFO[t]
    if cols % bs:
        raise ValueError(f"row length {cols} is not a multiple of block size {bs} for {name}")
    return cols // bs * ts
