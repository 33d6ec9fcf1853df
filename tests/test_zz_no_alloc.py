"""lmc_attention_decode_noalloc: the attention entry point for callers that
cannot allocate device memory where they decode (graph capture, loops that
must not synchronize on cudaMalloc/cudaFree, hosts owning all device
memory).  Called through the C ABI, it must match lmc_attention_decode with
a caller workspace and the oracle's attention read, on two calls in a row
(the fixed scratch array keeps the previous call's contents, which must not
leak into the next result).

Kept in a file pytest collects last, so a stop-at-first-failure run has
already run every other test."""
import numpy as np
import pytest

from lmc_b200 import runtime as rt
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


def _case(torch, seed, H, Hkv, Dh, S, pos, B):
    rng = np.random.default_rng(seed)
    kc = rng.normal(0, 1, (B, Hkv, S, Dh)).astype(np.float32)
    vc = rng.normal(0, 1, (B, Hkv, S, Dh)).astype(np.float32)
    q = rng.normal(0, 1, (B, H * Dh)).astype(np.float32)
    kn = rng.normal(0, 1, (B, Hkv * Dh)).astype(np.float32)
    vn = rng.normal(0, 1, (B, Hkv * Dh)).astype(np.float32)
    poss = np.array([pos - b for b in range(B)], np.int32)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return dict(kc=d(kc), vc=d(vc), q=d(q), kn=d(kn), vn=d(vn), pos=d(poss))


def _run(torch, t, H, Hkv, Dh, S, B, noalloc):
    out = torch.empty((B, H * Dh), dtype=torch.float32, device="cuda")
    kc, vc = t["kc"].clone(), t["vc"].clone()
    args = [out.data_ptr(), t["q"].data_ptr(), t["kn"].data_ptr(), t["vn"].data_ptr(), kc.data_ptr(),
            vc.data_ptr(), rt.KV_F32, t["pos"].data_ptr(), B, H, Hkv, Dh, S]
    if noalloc:
        rt.call("lmc_attention_decode_noalloc", *args, None)
    else:
        wsb = rt.lib().lmc_attention_workspace_bytes(B, H, Dh, S)
        ws = torch.empty(max(wsb, 4), dtype=torch.uint8, device="cuda")
        rt.call("lmc_attention_decode", *args, ws.data_ptr(), wsb, None)
    torch.cuda.synchronize()
    return out.cpu().numpy(), kc.cpu().numpy()


# The second call's position lies several context splits below the first's,
# so the splits the first call filled are empty in the second: leftovers of
# the first call in the shared array must not reach the second result.
@pytest.mark.parametrize("H,Hkv,Dh,S,pos,pos2,B",
                         [(12, 12, 64, 1024, 700, 90, 2), (32, 8, 128, 4096, 3000, 200, 1)])
def test_noalloc_matches_workspace_entry(cuda, orc, H, Hkv, Dh, S, pos, pos2, B):
    for call, (seed, p) in enumerate(((11, pos), (12, pos2))):  # two calls in a row, different data
        t = _case(cuda, seed, H, Hkv, Dh, S, p, B)
        want, kc_want = _run(cuda, t, H, Hkv, Dh, S, B, noalloc=False)
        got, kc_got = _run(cuda, t, H, Hkv, Dh, S, B, noalloc=True)
        assert rel_err(got, want) < 1e-5, f"call {call}"
        assert np.array_equal(kc_got, kc_want)
        # and the oracle's attention read over the cache the call wrote
        for b in range(B):
            ref = orc.attention(t["q"][b].cpu().numpy(), kc_got[b], _vc_after(t, b), H, Hkv, Dh, S, p - b)
            assert rel_err(got[b], ref) < 1e-5, f"call {call} row {b} vs oracle"


def _vc_after(t, b):
    """The V cache of row b after the call: the new V row at its position."""
    vc = t["vc"][b].cpu().numpy().copy()
    pos = int(t["pos"][b].item())
    Hkv, Dh = vc.shape[0], vc.shape[2]
    vc[:, pos, :] = t["vn"][b].cpu().numpy().reshape(Hkv, Dh)
    return vc


def test_noalloc_rejects_oversized_shape(cuda):
    B, H, Dh, S = 64, 64, 256, 65536  # needs far more than the fixed scratch
    assert rt.lib().lmc_attention_workspace_bytes(B, H, Dh, S) > (4 << 20)
    x = cuda.zeros(16, device="cuda")
    p = cuda.zeros(B, dtype=cuda.int32, device="cuda")
    with pytest.raises(rt.LmcError) as e:
        rt.call("lmc_attention_decode_noalloc", x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(),
                x.data_ptr(), x.data_ptr(), rt.KV_F32, p.data_ptr(), B, H, H, Dh, S, None)
    assert e.value.code == -1 and "fixed" in str(e.value)
