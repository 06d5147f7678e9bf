"""Writes prng_vectors.json from a pure-Python restatement of PRNGKey
(jax-rs 0.5.1 src/random.rs:29-97,161-210): xorshift128+ on u64 with
wrapping arithmetic.  It is independent of the C oracle, so the test that
compares the two pins the oracle's integer stream and its exact f32 uniforms.
Run: python tests/golden/make_prng_vectors.py
"""
import json
import os

M64 = (1 << 64) - 1


def from_seed(seed):
    return [seed & M64, (seed * 0x9E3779B97F4A7C15) & M64]


def rotl(x, r):
    return ((x << r) | (x >> (64 - r))) & M64


def rotr(x, r):
    return ((x >> r) | (x << (64 - r))) & M64


def split(k):
    a = [(k[0] + 0x9E3779B97F4A7C15) & M64, rotl(k[1], 27)]
    b = [(k[0] + 0x3C6EF372FE94F82A) & M64, rotr(k[1], 17)]
    return a, b


def next_u64(k):
    s1, s0 = k[0], k[1]
    k[0] = s0
    s1 ^= (s1 << 23) & M64
    s1 ^= s1 >> 17
    s1 ^= s0
    s1 ^= s0 >> 26
    k[1] = s1
    return (s1 + s0) & M64


def main():
    vec = {"reference": "jax-rs 0.5.1 src/random.rs", "cases": []}
    for seed in (0, 1, 2, 3, 42):
        k = from_seed(seed)
        a, b = split(k)
        ka = list(a)
        u64 = [next_u64(ka) for _ in range(8)]
        kb = list(b)
        # next_f32: (u >> 40) / 2^24 is exact in f32; stored as the 24-bit numerator
        f24 = [next_u64(kb) >> 40 for _ in range(8)]
        kr = list(b)
        randint10 = [next_u64(kr) % 10 for _ in range(8)]
        vec["cases"].append({"seed": seed, "key": [hex(x) for x in k], "split0": [hex(x) for x in a],
                             "split1": [hex(x) for x in b], "u64_from_split0": [hex(x) for x in u64],
                             "f32_numerators_from_split1": f24, "randint_0_10_from_split1": randint10})
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "prng_vectors.json")
    with open(out, "w") as f:
        json.dump(vec, f, indent=1)
    print(out)


if __name__ == "__main__":
    main()
