"""The measurement reference p2p_debug_stream_read: it reads every byte it is given once (its
XOR checksum equals numpy's) and refuses unaligned arguments."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import p2p_b200
    c = p2p_b200.Context(0)
    yield c
    c.close()


@pytest.mark.parametrize("nbytes", [16, 4096 + 48, 8 * 2**20 + 16 * 37, 200 * 2**20])
def test_stream_read_checksum(ctx, nbytes):
    g = torch.Generator(device="cuda").manual_seed(nbytes)
    words = torch.randint(-2**31, 2**31 - 1, (nbytes // 4 + 64,), generator=g, device="cuda",
                          dtype=torch.int32)
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    ctx.debug_stream_read(words, out, nbytes)
    torch.cuda.synchronize()
    want = np.bitwise_xor.reduce(words[: nbytes // 4].cpu().numpy().view(np.uint32))
    assert int(out.cpu().numpy().view(np.uint32)[0]) == int(want)


def test_stream_read_rejects_unaligned(ctx):
    import p2p_b200
    words = torch.zeros(1024, dtype=torch.int32, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(p2p_b200.P2PError):
        ctx.debug_stream_read(words, out, 100)  # not a multiple of 16
    with pytest.raises(p2p_b200.P2PError):
        ctx.debug_stream_read(words[1:], out, 64)  # 4-byte aligned source
