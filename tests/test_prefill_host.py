"""Host-side index arithmetic of the paged prefill (csrc/attn.cu,
launch_paged_centroids), on CPU: a chunk of n tokens starting at first_pos
must compute the centroid of exactly the blocks whose last token (16 lb + 15)
it wrote -- the blocks [first_pos / 16, (first_pos + n) / 16)."""


def centroid_blocks(first_pos, n):
    return list(range(first_pos // 16, (first_pos + n) // 16))


def test_centroid_range_matches_brute_force():
    for first_pos in range(0, 200):
        for n in range(1, 90):
            want = [lb for lb in range(0, 40) if first_pos <= 16 * lb + 15 < first_pos + n]
            assert centroid_blocks(first_pos, n) == want, (first_pos, n)


def test_chunks_cover_every_block_once():
    # a prompt split into chunks of any size computes each full block once
    for prompt in (1, 15, 16, 100, 2048):
        for rows in (1, 3, 8, 64):
            seen = []
            for c0 in range(0, prompt, rows):
                seen += centroid_blocks(c0, min(rows, prompt - c0))
            assert seen == list(range(prompt // 16)), (prompt, rows)
