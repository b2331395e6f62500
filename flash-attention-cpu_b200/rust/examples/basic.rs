//! The crate's API on the GPU: one head (plain and causal), a batched
//! multi-head call, the three schedules agreeing, and the CPU naive oracle.
use flash_attention_cpu::{flash_attention, flash_attention_multihead, flash_attention_v1,
                          flash_attention_v3, naive, FlashAttentionConfig};

/// Deterministic values in (-1, 1) from a 64-bit mixing sequence.
fn values(n: usize, seed: u64) -> Vec<f32> {
    let mut s = seed ^ 0x5DEECE66D;
    (0..n)
        .map(|_| {
            s = s.wrapping_mul(6364136223846793005).wrapping_add(1442695040888963407);
            ((s >> 40) as f32 / (1u64 << 24) as f32) * 2.0 - 1.0
        })
        .collect()
}

fn max_diff(a: &[f32], b: &[f32]) -> f32 {
    a.iter().zip(b).map(|(x, y)| (x - y).abs()).fold(0.0, f32::max)
}

fn main() {
    let (s, d) = (256usize, 64usize);
    let (q, k, v) = (values(s * d, 1), values(s * d, 2), values(s * d, 3));
    let mut out = vec![0.0f32; s * d];
    let mut want = vec![0.0f32; s * d];

    flash_attention(&q, &k, &v, s, s, d, &FlashAttentionConfig::default(), &mut out);
    naive::naive_attention(&q, &k, &v, s, s, d, false, &mut want);
    println!("single head: out[0][..4] = {:?}, max |gpu - naive| = {:e}", &out[..4],
             max_diff(&out, &want));

    let causal = FlashAttentionConfig { causal: true, ..Default::default() };
    flash_attention(&q, &k, &v, s, s, d, &causal, &mut out);
    println!("causal: row 0 equals V row 0 to {:e}", max_diff(&out[..d], &v[..d]));

    let (b, h) = (4usize, 8usize);
    let n = b * h * s * d;
    let (mq, mk, mv) = (values(n, 4), values(n, 5), values(n, 6));
    let mut mo = vec![0.0f32; n];
    flash_attention_multihead(&mq, &mk, &mv, b, h, s, s, d, &causal, &mut mo);
    println!("multihead [{b}, {h}, {s}, {d}]: out[0][..4] = {:?}", &mo[..4]);

    let mut o1 = vec![0.0f32; s * d];
    let mut o3 = vec![0.0f32; s * d];
    flash_attention_v1(&q, &k, &v, s, s, d, &causal, &mut o1);
    flash_attention_v3(&q, &k, &v, s, s, d, &causal, &mut o3);
    println!("v1 vs v3: max diff {:e}", max_diff(&o1, &o3));
}
