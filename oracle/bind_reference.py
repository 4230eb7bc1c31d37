"""TEST INFRASTRUCTURE ONLY: writes the reference's src/nn/layer.cpp with the
B200 dispatch a maintainer would add (oracle/binding/cuda_spec_backend.hpp)
into a build folder (oracle/_ref/bind/, git-ignored).  Two calls go in, each
at the top of its method, after the line that reads the model's backend:

  TransformerDecoder::generate_speculative (src/nn/layer.cpp:1382-1386)
  TransformerDecoder::generate_advanced    (src/nn/layer.cpp:1240-1244)

and the binding header after the file's own includes.  Nothing else of the
file changes; the script stops if an anchor is not where it expects.

    python oracle/bind_reference.py <reference>/src/nn/layer.cpp oracle/_ref/bind/layer.cpp
"""
import os
import sys

BACKEND_LINE = "auto backend = token_emb_->parameters()[0]->backend();"

SPEC = """  if (std::vector<size_t> cuda_out;
      cuda_spec_dispatch_speculative(this, backend, draft_model, prompt, max_new_tokens, lookahead, temperature,
                                     top_k, top_p, seed, quantized_cache, &cuda_out))
    return cuda_out;
"""
ADV = """  if (std::vector<size_t> cuda_out;
      cuda_spec_dispatch_advanced(this, backend, prompt, max_new_tokens, temperature, top_k, top_p, seed,
                                  use_kv_cache, &cuda_out))
    return cuda_out;
"""


def insert_after_backend(lines, signature, block):
    start = next((i for i, l in enumerate(lines) if signature in l), None)
    if start is None:
        raise SystemExit(f"anchor not found: {signature}")
    for i in range(start, min(start + 12, len(lines))):
        if BACKEND_LINE in lines[i]:
            lines.insert(i + 1, block)
            return
    raise SystemExit(f"backend line not found after {signature}")


def main(src, dst):
    with open(src) as f:
        lines = f.readlines()
    last_inc = max(i for i, l in enumerate(lines) if l.startswith("#include"))
    lines.insert(last_inc + 1, '#include "cuda_spec_backend.hpp"\n')
    insert_after_backend(lines, "TransformerDecoder::generate_speculative(", SPEC)
    insert_after_backend(lines, "TransformerDecoder::generate_advanced(", ADV)
    os.makedirs(os.path.dirname(dst), exist_ok=True)
    with open(dst, "w") as f:
        f.writelines(lines)


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2])
