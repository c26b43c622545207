"""Write tests/golden/bundle_ref/, an encoder bundle saved by the reference's
own save_encoders (src/prismkv/weights.py:18-36), so that tests can check
that this library loads the reference's format.

Run in a container that has the reference checkout (read-only):

    PRISMKV_REFERENCE=/path/to/reference python tests/golden/make_bundle.py

Two (layer, KV group) encoders of SharedSAE(head_dim=8, features=16) with
seeded weights and distinct scales; the metadata records the torch version.
"""
import json
import os
import shutil
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("PRISMKV_REFERENCE", "/root/reference"))
sys.path.insert(0, str(REF / "src"))
from prismkv.core import SharedSAE  # noqa: E402
from prismkv.hf_reference import Encoder  # noqa: E402
from prismkv.weights import save_encoders  # noqa: E402

OUT = HERE / "bundle_ref"


def main():
    torch.manual_seed(1234)
    bundle = {}
    for (layer, group, ks, qs) in ((0, 1, 1.5, 0.75), (3, 0, 2.0, 1.25)):
        sae = SharedSAE(8, 16, 2, 4)
        with torch.no_grad():
            sae.W_enc.copy_(torch.randn(16, 8) / 8 ** 0.5)
            sae.b_enc.copy_(0.01 * torch.randn(16))
        bundle[(layer, group)] = Encoder(sae, ks, qs)
    if OUT.exists():
        shutil.rmtree(OUT)
    save_encoders(bundle, OUT, metadata={"generator": "tests/golden/make_bundle.py", "torch": torch.__version__})
    # The expected tensors, for the loading test.
    expect = {f"{l},{g}": dict(W=e.sae.W_enc.detach().tolist(), b=e.sae.b_enc.detach().tolist(),
                               key_scale=e.key_scale, query_scale=e.query_scale)
              for (l, g), e in bundle.items()}
    (HERE / "bundle_ref_expect.json").write_text(json.dumps(expect))
    print("wrote", OUT)


if __name__ == "__main__":
    main()
