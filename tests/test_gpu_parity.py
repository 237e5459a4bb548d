"""GPU parity of the B200 codec against the CPU oracle, through the C ABI.

Bar (per the codec's contract):
  * bitmap and dominant-sign bits bit-exact,
  * residual / stats bit-exact in raw mode ("sz3_memcpy"),
  * q8 / int4 codes within +-1 LSB (and in practice identical),
  * decoded update relative L2 <= 1e-6 against the oracle's decoder.
The oracle is the C restatement (oracle/falcom_oracle.c), itself pinned
bit-exact against the reference build in tests/test_oracle_*.py.  The same
encoder/decoder cases run on the CPU against the kernel emulator in
tests/test_kernel_emulation.py.
"""
import numpy as np
import pytest

from compressor_b200.abi import Codec
from oracle import binding as ob
from tests.helpers import frame_content, seeded
from tests.parity_cases import SHAPES, THRESHOLD, check_encoder_decoder, make_rounds

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("codec", ["raw", "q8", "int4", "q8_raw", "int4_raw"])
def test_encoder_decoder_match_oracle(product_lib, codec):
    check_encoder_decoder(product_lib, codec)


def test_against_reference_build_raw(product_lib):
    """Same seeded batches through the reference library (built from the
    reference's own sources) and through this codec in raw mode."""
    if not ob.have_ref():
        pytest.skip("reference build oracle/_ref not present")
    ours = Codec(product_lib, client="client_0", param_count_threshold=THRESHOLD)
    ref = Codec(ob.REF_SO, client="client_0", param_count_threshold=THRESHOLD)
    ours_d = Codec(product_lib, client="client_0", param_count_threshold=THRESHOLD)
    ref_d = Codec(ob.REF_SO, client="client_0", param_count_threshold=THRESHOLD)
    ours.lib.falcom_set_residual_codec(ours.h, b"raw")
    names = [n for n, _ in SHAPES]
    for t, xs in enumerate(make_rounds(4, seed=5)):
        r1, A, _ = ours.compress_batch(names, xs)
        r2, B, _ = ref.compress_batch(names, xs)
        assert r1 == 0 and r2 == 0
        for a, b in zip(A, B):
            assert (a.type, a.step, a.shape, a.original_dtype, a.stored_dtype) == (
                b.type, b.step, b.shape, b.original_dtype, b.stored_dtype)
            if a.codec == "sz3_memcpy":
                assert b.codec == "sz3_memcpy" and a.data == b.data
            else:
                assert frame_content(a.data) == frame_content(b.data)
            assert frame_content(a.bitmap) == frame_content(b.bitmap)
            assert frame_content(a.dominant_signs) == frame_content(b.dominant_signs)
            assert (a.current_mean, a.current_std, a.prev_mean, a.prev_std, a.global_min,
                    a.global_max, a.num_predicted_kernels, a.prediction_ratio,
                    a.sign_mismatch_ratio) == (
                b.current_mean, b.current_std, b.prev_mean, b.prev_std, b.global_min,
                b.global_max, b.num_predicted_kernels, b.prediction_ratio, b.sign_mismatch_ratio)
        # cross decode: each decoder reads the other's payloads
        ra, YA = ours_d.decompress_batch(names, B)
        rb, YB = ref_d.decompress_batch(names, A)
        assert ra == 0 and rb == 0
        for ya, yb in zip(YA, YB):
            assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32))


def test_libzstd_frames_byte_identical_to_reference(product_lib):
    if not ob.have_ref():
        pytest.skip("reference build oracle/_ref not present")
    ours = Codec(product_lib, client="client_0", param_count_threshold=THRESHOLD)
    ref = Codec(ob.REF_SO, client="client_0", param_count_threshold=THRESHOLD)
    ours.lib.falcom_set_residual_codec(ours.h, b"raw")
    assert ours.lib.falcom_set_frame_mode(ours.h, b"libzstd") == 0
    names = [n for n, _ in SHAPES]
    for xs in make_rounds(3, seed=9):
        _, A, _ = ours.compress_batch(names, xs)
        _, B, _ = ref.compress_batch(names, xs)
        for a, b in zip(A, B):
            assert a.bitmap == b.bitmap
            assert a.dominant_signs == b.dominant_signs
            assert a.data == b.data
            size_a = len(a.data) + len(a.bitmap) + len(a.dominant_signs)
            size_b = len(b.data) + len(b.bitmap) + len(b.dominant_signs)
            assert size_a == size_b   # compression ratio identical


def test_gpu_frames_are_valid_zstd(product_lib):
    c = Codec(product_lib, client="c", param_count_threshold=THRESHOLD)
    names = ["big.weight", "ones.weight"]
    xs0 = [seeded((256, 256, 3, 3), 1), np.ones((1024, 300, 1, 1), np.float32)]
    xs1 = [seeded((256, 256, 3, 3), 2), np.ones((1024, 300, 1, 1), np.float32)]
    c.compress_batch(names, xs0)
    _, L, _ = c.compress_batch(names, xs1)
    for layer in L:
        bm = ob.zstd_decompress(layer.bitmap)
        assert len(bm) == (layer.shape[0] * layer.shape[1] + 7) // 8
    # all-ones bitmap of 1x1 kernels: RLE blocks keep the frame tiny
    assert len(L[1].bitmap) < 64
