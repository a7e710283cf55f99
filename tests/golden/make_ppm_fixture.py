"""Pack the reference's network-validation images into a fixture.

The reference validates whole networks on four real images
(tests/validate_network.py:15-38 make_batch: tests/samples/{cat,dog,parrot,
goldfish}.ppm, 224x224 P6, labels 281, 207, 87, 1).  The reference tree does
not travel to the machines that run the GPU tests, so this script reads the
PPM files where the reference lies and stores their raw RGB bytes, unchanged,
as one uint8 tensor:

    python tests/golden/make_ppm_fixture.py [reference root]

ppm_samples.pt: {"images": uint8 [4, 224, 224, 3] (HWC, as in the files),
                 "labels": int64 [4], "names": [...], "source": "..."}
The ImageNet normalisation of make_batch is applied by the test that loads
the fixture.
"""
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
SAMPLES = {"cat": 281, "dog": 207, "parrot": 87, "goldfish": 1}  # validate_network.py:21


def read_ppm(path):
    """Binary PPM (P6, maxval 255): header tokens then width*height*3 bytes."""
    with open(path, "rb") as f:
        data = f.read()
    tokens, pos = [], 0
    while len(tokens) < 4:
        while data[pos:pos + 1].isspace():
            pos += 1
        if data[pos:pos + 1] == b"#":  # comment to end of line
            while data[pos:pos + 1] not in (b"\n", b""):
                pos += 1
            continue
        start = pos
        while not data[pos:pos + 1].isspace():
            pos += 1
        tokens.append(data[start:pos])
    pos += 1  # the single whitespace byte after maxval
    magic, w, h, maxval = tokens[0], int(tokens[1]), int(tokens[2]), int(tokens[3])
    if magic != b"P6" or maxval != 255:
        raise ValueError(f"{path}: not an 8-bit P6 image")
    pix = data[pos:pos + w * h * 3]
    if len(pix) != w * h * 3:
        raise ValueError(f"{path}: truncated pixel data")
    return torch.frombuffer(bytearray(pix), dtype=torch.uint8).reshape(h, w, 3)


def main(argv):
    root = argv[1] if len(argv) > 1 else "/root/reference"
    src = os.path.join(root, "tests", "samples")
    imgs = [read_ppm(os.path.join(src, n + ".ppm")) for n in SAMPLES]
    out = {"images": torch.stack(imgs), "labels": torch.tensor(list(SAMPLES.values()), dtype=torch.int64),
           "names": list(SAMPLES), "source": "reference tests/samples/*.ppm (validate_network.py make_batch)"}
    torch.save(out, os.path.join(HERE, "ppm_samples.pt"))
    print("wrote ppm_samples.pt", tuple(out["images"].shape))


if __name__ == "__main__":
    main(sys.argv)
