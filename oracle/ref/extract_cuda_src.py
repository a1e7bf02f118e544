"""Build step of the reference comparator (test infrastructure only).

h3-rs keeps its CUDA C kernels as Rust raw-string constants (`const SRC: &str = r#"..."#;`) that it compiles
with NVRTC at run time (kernels.rs:12-528, attn8.rs:12-346).  This script copies that text out of the
reference's .rs file into a .cu file under oracle/_ref/ (git-ignored build output) so nvcc can compile the
reference's own kernels for sm_100a as a GPU comparator.  Nothing it writes is committed.

usage: extract_cuda_src.py <file.rs> <out.cu>
"""
import sys


def extract(rs_text: str) -> str:
    start_tok = 'const SRC: &str = r#"'
    i = rs_text.index(start_tok) + len(start_tok)
    j = rs_text.index('"#;', i)
    return rs_text[i:j]


def main() -> None:
    src, dst = sys.argv[1], sys.argv[2]
    with open(src, encoding="utf-8") as f:
        body = extract(f.read())
    with open(dst, "w", encoding="utf-8") as f:
        f.write(f"// extracted at build time from {src.split('/src/')[-1]} (not committed)\n")
        f.write(body)


if __name__ == "__main__":
    main()
