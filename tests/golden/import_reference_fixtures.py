"""Copy the reference's block golden vectors into ``tests/golden/{rb,tf}``.

The reference ships two PyTorch-generated known-answer fixtures as raw fp16
files (``app/src/main/assets/rb`` — one ResnetBlock2D at C=320, 64x64, temb
1280; ``app/src/main/assets/tf`` — one Transformer2DModel block at C=320,
64x64, context 77x768, 8 heads; consumed by ``VulkanBench.kt:39-64`` and
``vk_engine.cpp:423-480,931-1012``). They are data, not source; they are
copied byte-for-byte so that tests can run where the reference checkout is not
mounted, and ``MANIFEST.txt`` records each file's size and sha256.

Usage: ``python tests/golden/import_reference_fixtures.py <reference-root>``
"""
import hashlib
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref_root: str) -> None:
    lines = []
    for sub in ("rb", "tf"):
        src = os.path.join(ref_root, "app", "src", "main", "assets", sub)
        dst = os.path.join(HERE, sub)
        os.makedirs(dst, exist_ok=True)
        for name in sorted(os.listdir(src)):
            if not name.endswith(".bin"):
                continue
            shutil.copyfile(os.path.join(src, name), os.path.join(dst, name))
            data = open(os.path.join(dst, name), "rb").read()
            lines.append(f"{sub}/{name} {len(data)} {hashlib.sha256(data).hexdigest()}")
    with open(os.path.join(HERE, "MANIFEST.txt"), "w") as f:
        f.write("\n".join(lines) + "\n")
    print("\n".join(lines))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: import_reference_fixtures.py <reference-root>")
    main(sys.argv[1])
