"""Regenerate the golden fixtures under tests/golden from the reference tree.

Run in a container where the reference checkout is mounted (read-only):

    python tests/golden/make_fixtures.py /root/reference

It copies the tiny checkpoints the reference's own GPU tests load
(tests/fixtures/tiny_*: config.json + model.safetensors, data only) and
extracts, from the reference test sources read as text, the numeric goldens
that pin the path:

* kOracle greedy ids            tests/test_engine_gpu.c:21-23
* qwen3_5 first-8 logits/argmax  tests/test_qwen3_5_goldens_gpu.c:14-30
* llama3 RoPE frequency vector   tests/test_rope_llama3.c:173-224
* llama3 config fixture          tests/fixtures/model_config_llama3/config.json

Nothing at test time reads the reference tree; the GPU box only sees the
files written here.
"""
import json
import os
import re
import shutil
import sys

FIXTURES = ["tiny_qwen3", "tiny_qwen3_tied", "tiny_qwen3_5", "tiny_qwen3_5_tied",
            "tiny_llama3", "tiny_llama3_tied", "tiny_mistral", "tiny_mistral_tied"]


def c_array(src, name):
    m = re.search(r"%s\s*\[\s*\d*\s*\]\s*=\s*\{(.*?)\};" % re.escape(name), src, re.S)
    if not m:
        raise SystemExit("array %s not found" % name)
    body = re.sub(r"/\*.*?\*/", "", m.group(1), flags=re.S)
    return [float(t.strip().rstrip("f")) for t in body.split(",") if t.strip()]


def c_int(src, name):
    m = re.search(r"%s\s*=\s*(-?\d+)\s*;" % re.escape(name), src)
    if not m:
        raise SystemExit("int %s not found" % name)
    return int(m.group(1))


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    out = os.path.dirname(os.path.abspath(__file__))
    for d in FIXTURES:
        dst = os.path.join(out, d)
        os.makedirs(dst, exist_ok=True)
        for f in ("config.json", "model.safetensors"):
            shutil.copyfile(os.path.join(ref, "tests", "fixtures", d, f), os.path.join(dst, f))
    os.makedirs(os.path.join(out, "model_config_llama3"), exist_ok=True)
    shutil.copyfile(os.path.join(ref, "tests/fixtures/model_config_llama3/config.json"),
                    os.path.join(out, "model_config_llama3", "config.json"))

    eng = open(os.path.join(ref, "tests/test_engine_gpu.c")).read()
    q35 = open(os.path.join(ref, "tests/test_qwen3_5_goldens_gpu.c")).read()
    rope = open(os.path.join(ref, "tests/test_rope_llama3.c")).read()
    goldens = {
        "kOracle": {"fixture": "tiny_qwen3", "prompt": [1, 2], "max_tokens": 8,
                    "ids": [int(v) for v in c_array(eng, "kOracle")],
                    "source": "tests/test_engine_gpu.c:21-23"},
        "qwen3_5_dense": {"fixture": "tiny_qwen3_5", "ids": [1, 2, 3, 4, 5],
                          "first8": c_array(q35, "dense_first8"),
                          "argmax": c_int(q35, "dense_argmax"), "atol": 1e-2,
                          "source": "tests/test_qwen3_5_goldens_gpu.c:18-22,119-123"},
        "qwen3_5_tied": {"fixture": "tiny_qwen3_5_tied", "ids": [1, 2, 3, 4, 5],
                         "first8": c_array(q35, "tied_first8"),
                         "argmax": c_int(q35, "tied_argmax"), "atol": 5e-2,
                         "source": "tests/test_qwen3_5_goldens_gpu.c:24-30,125-129"},
        "llama3_freqs": {"config": "model_config_llama3", "head_dim": 128,
                         "freqs": c_array(rope, "golden"), "rtol": 1e-5,
                         "source": "tests/test_rope_llama3.c:173-224"},
    }
    with open(os.path.join(out, "goldens.json"), "w") as f:
        json.dump(goldens, f, indent=1)
    print("wrote fixtures to", out)


if __name__ == "__main__":
    main()
