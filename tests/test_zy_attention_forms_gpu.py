"""The non-default attention forward forms against the fp32 statement.  The
form is fixed per process (SHIFT_ATTN_FWD is read once), so each runs in a
child process."""
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("form", ["split_fma", "fold", "tmem"])
def test_attention_forward_forms_in_a_fresh_process(form):
    """Output of the form against the fp32 statement, with keys scaled up along
    the sequence so that rows' maxima grow across key blocks (the rescale
    paths run)."""
    import os
    import subprocess
    import sys
    code = (
        "import math, torch\n"
        "from shift_b200.ops import functional as Fn\n"
        "from shift_b200.ops import reference as ref\n"
        "torch.manual_seed(3)\n"
        "B, S, Hq, Hkv, D = 2, 1024, 8, 2, 64\n"
        "T = B * S\n"
        "x = torch.randn(T, (Hq + 2 * Hkv) * D, device='cuda')\n"
        "pos = torch.arange(S, device='cuda').repeat(B).float()\n"
        "x[:, Hq * D:(Hq + Hkv) * D] *= (1.0 + 6.0 * pos / S)[:, None]\n"
        "qkv = x.to(torch.bfloat16)\n"
        "scale = 1 / math.sqrt(D)\n"
        "o, lse = Fn.attention_fwd(qkv, B, S, Hq, Hkv, D, scale)\n"
        "f = qkv.float()\n"
        "q = f[:, :Hq * D].view(T, Hq, D); k = f[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)\n"
        "v = f[:, (Hq + Hkv) * D:].view(T, Hkv, D)\n"
        "want = ref.attention(q, k, v, B, S, scale).reshape(T, Hq * D)\n"
        "err = (o.float() - want).abs().max().item() / (want.abs().max().item() + 1e-6)\n"
        "torch.cuda.synchronize()\n"
        "print('ERR', err)\n"
        "assert err <= 2e-2, err\n"
    )
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, SHIFT_ATTN_FWD=form, PYTHONPATH=root + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
