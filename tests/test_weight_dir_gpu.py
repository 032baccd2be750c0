"""The reference's weight-directory format as a drop-in (``unet_w/<key>.bin``).

The reference reads each UNet tensor lazily from ``<dir>/<key>.bin``: raw
little-endian fp16, Linear weights stored ``[in, out]`` (``vk_engine.cpp:497-507``,
``README.md:293,297``). Here the seeded weights are written in that layout,
loaded through ``sdg_init(device, dir)`` and through ``sdg_load_dir``, and the
forward must be bit-identical to the engine that received the same tensors
through ``sdg_upload_weight``. A damaged directory must fail with
``SDG_ERR_IO`` naming the file (the reference substitutes zeros, ``:500-503``).
"""
import os

import numpy as np
import pytest

from oracle import weights as W

pytestmark = pytest.mark.gpu
SDG_ERR_IO = 6


@pytest.fixture(scope="module")
def weight_dir(tmp_path_factory, unet_weights):
    d = tmp_path_factory.mktemp("unet_w")
    for key, arr in W.iter_reference_blobs(unet_weights):
        arr.tofile(os.path.join(d, key + ".bin"))
    return str(d)


def _inputs():
    lat, t, ctx = W.make_inputs(2, 16, 16, seed=7)
    return lat.numpy(), t.numpy(), ctx.numpy()


def test_init_from_dir_and_load_dir_match_upload(sdg, engine, weight_dir):
    lat, t, ctx = _inputs()
    ref = engine.forward(lat, t, ctx)
    e1 = sdg.Engine(0, weights_dir=weight_dir)          # sdg_init(device, dir)
    try:
        e1.prepare()
        got1 = e1.forward(lat, t, ctx)
    finally:
        e1.release()
    e2 = sdg.Engine(0)                                  # sdg_init(device, NULL) + sdg_load_dir
    try:
        e2.load_dir(weight_dir)
        e2.prepare()
        got2 = e2.forward(lat, t, ctx)
    finally:
        e2.release()
    assert np.isfinite(ref).all()
    assert np.array_equal(got1, ref)
    assert np.array_equal(got2, ref)


def _damaged_copy(src, dst, key, keep_bytes):
    os.makedirs(dst, exist_ok=True)
    for name in os.listdir(src):
        data = open(os.path.join(src, name), "rb").read()
        if name == key + ".bin":
            data = data[:keep_bytes]
        open(os.path.join(dst, name), "wb").write(data)


def test_truncated_weight_file_is_an_io_error(sdg, cuda, weight_dir, tmp_path):
    key = "down_blocks.1.resnets.0.conv1.weight"
    size = os.path.getsize(os.path.join(weight_dir, key + ".bin"))
    # cut to a whole number of fp16 values: load succeeds, preparation reports the file and the key
    d1 = str(tmp_path / "short")
    _damaged_copy(weight_dir, d1, key, size // 2)
    e = sdg.Engine(0)
    try:
        e.load_dir(d1)
        with pytest.raises(sdg.SdgError) as ei:
            e.prepare()
        assert ei.value.code == SDG_ERR_IO
        assert key in str(ei.value) and "truncated" in str(ei.value)
    finally:
        e.release()
    # cut to an odd byte count: not fp16 data at all, refused while reading the directory
    d2 = str(tmp_path / "odd")
    _damaged_copy(weight_dir, d2, key, size // 2 + 1)
    with pytest.raises(sdg.SdgError) as ei:
        sdg.Engine(0, weights_dir=d2)
    assert ei.value.code == SDG_ERR_IO and key in str(ei.value)
