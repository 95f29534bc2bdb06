"""Generates tests/golden/kat.json: known-answer vectors for the hot path.

The reference ships no numeric golden tensors, so these are authored from
its source:
  * nibble/byte order: Sources/NovaMLXEngine/FusedQuantizedSDPA.swift:79-81
    (value d of a row sits in word d / (32/bits) at bit (d % (32/bits))*bits);
  * quantization: the workload rule (scale = (max-min)/(2^bits-1), bias = min,
    q = round-half-even((w-bias)/scale)); the cases are built so every
    expected code is an exact small integer and is written out literally;
  * block hashes: BlockHasher.computeBlockHash's byte layout
    (Sources/NovaMLXPrefixCache/BlockHasher.swift:7-27), hashed here with
    Python's hashlib, independently of the C++ SHA-1 in the library.
Run: python tests/golden/gen_golden.py
"""
import hashlib
import json
import struct
from pathlib import Path

OUT = Path(__file__).resolve().parent / "kat.json"


def block_hash(parent, tokens, model_name):
    h = hashlib.sha1()
    if model_name:
        h.update(model_name.encode())
    h.update(parent if parent is not None else b"NovaMLX-root")
    h.update(struct.pack("<q", len(tokens)))
    for t in tokens:
        h.update(struct.pack("<i", t))
    return h.digest()


def chain(tokens, bs, model):
    out, parent = [], None
    for i in range(len(tokens) // bs):
        parent = block_hash(parent, tokens[i * bs:(i + 1) * bs], model)
        out.append(parent.hex())
    return out


def main():
    kat = {}
    kat["nibble"] = [
        {"bits": 4, "word": 0x76543210, "values": [0, 1, 2, 3, 4, 5, 6, 7]},
        {"bits": 4, "word": 0xFEDCBA98, "values": [8, 9, 10, 11, 12, 13, 14, 15]},
        {"bits": 4, "word": 0x0000000F, "values": [15, 0, 0, 0, 0, 0, 0, 0]},
        {"bits": 4, "word": 0xF0000000, "values": [0, 0, 0, 0, 0, 0, 0, 15]},
        {"bits": 8, "word": 0x04030201, "values": [1, 2, 3, 4]},
        {"bits": 8, "word": 0xFF00AA55, "values": [0x55, 0xAA, 0x00, 0xFF]},
    ]
    # one group of 64 per case; expected codes are exact integers
    ramp = [(i % 16) * 0.25 for i in range(64)]
    tie = [0.0, 15.0, 0.5, 1.5, 2.5, 3.5, 4.5, 5.5] + [0.0] * 56
    byte = [i * 4.0 for i in range(63)] + [255.0]
    kat["quantize"] = [
        {"bits": 4, "group": 64, "w": ramp, "q": [i % 16 for i in range(64)], "scale_f16": 0x3400, "bias_f16": 0},
        {"bits": 4, "group": 64, "w": [1.5] * 64, "q": [0] * 64, "scale_f16": 0, "bias_f16": 0x3E00},
        {"bits": 4, "group": 64, "w": tie, "q": [0, 15, 0, 2, 2, 4, 4, 6] + [0] * 56, "scale_f16": 0x3C00,
         "bias_f16": 0},
        {"bits": 8, "group": 64, "w": byte, "q": [i * 4 for i in range(63)] + [255], "scale_f16": 0x3C00,
         "bias_f16": 0},
        {"bits": 4, "group": 32, "w": ramp[:32] + [x + 1.0 for x in ramp[:32]],
         "q": [i % 16 for i in range(32)] * 2, "scale_f16": [0x3400, 0x3400], "bias_f16": [0, 0x3C00]},
    ]
    # qmatmul with exact answer: x = ones[64]; row = ramp → Σ = 4·(0+…+15)·0.25 = 120
    kat["qmatmul"] = {"bits": 4, "group": 64, "x": [1.0] * 64, "w_row": ramp, "rows": 16, "y": 120.0}
    kat["block_hash"] = [
        {"parent": None, "tokens": [1, 2, 3, 4, 5, 6, 7, 8], "model": "test-model",
         "hex": block_hash(None, [1, 2, 3, 4, 5, 6, 7, 8], "test-model").hex()},
        {"parent": None, "tokens": [1, 2, 3], "model": "", "hex": block_hash(None, [1, 2, 3], "").hex()},
        {"parent": block_hash(None, [10, 20], "test").hex(), "tokens": [1, 2, 3], "model": "test",
         "hex": block_hash(block_hash(None, [10, 20], "test"), [1, 2, 3], "test").hex()},
        {"parent": None, "tokens": [], "model": "m", "hex": block_hash(None, [], "m").hex()},
        {"parent": None, "tokens": [-1, 2147483647, 128255], "model": "llama",
         "hex": block_hash(None, [-1, 2147483647, 128255], "llama").hex()},
    ]
    kat["chain"] = {"tokens": list(range(256)), "block_size": 64, "model": "test",
                    "hex": chain(list(range(256)), 64, "test")}
    OUT.write_text(json.dumps(kat, indent=1) + "\n")
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
