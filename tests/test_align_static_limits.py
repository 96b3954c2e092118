"""Host-side checks of moe_align_static's documented size limit (no GPU: the
size check rejects a request before any CUDA call, and the workspace query
is host arithmetic). They keep the limit stated in include/moe_b200.h (and
the integration notes) tied to moe_align_workspace_size."""
from mail_b200 import _lib

STATIC_BYTES = 1 << 20  # MOE_ALIGN_STATIC_SCRATCH_BYTES
FAKE = 256  # never dereferenced: rejected requests return before touching memory


def ws(T, k, E):
    return _lib.load().moe_align_workspace_size(T, k, E, 128)


def test_documented_example_fits_and_next_size_is_rejected():
    # top-8 over 256 experts: 8192 tokens need about 0.5 MiB and fit,
    # 16288 tokens are the largest that fit, 16384 tokens need 1.005 MiB
    assert ws(8192, 8, 256) == 527_616
    assert ws(16288, 8, 256) <= STATIC_BYTES < ws(16289, 8, 256)
    assert ws(16384, 8, 256) == 1_053_952
    lib = _lib.load()
    rc = lib.moe_align_static(FAKE, 16384, 8, 256, 128, FAKE, FAKE, FAKE, FAKE, FAKE, None)
    assert rc == 1 and "scratch" in lib.moe_last_error().decode()


def test_one_cta_batches_need_no_scratch_within_the_limit():
    # every batch the one-CTA align takes (<= 16384 slots, <= 1024 experts)
    # is also within the static limit, so the limit only binds larger ones
    assert ws(16384 // 8, 8, 1024) <= STATIC_BYTES
    assert ws(16384, 1, 1024) <= STATIC_BYTES
