//! Textbook attention that materialises the whole `[seq_len_q, seq_len_k]`
//! score matrix: the crate's correctness oracle and benchmark comparison point
//! (src/naive.rs:14-75).  It stays CPU code in this crate; the GPU forward
//! never calls it.

/// `q`: `[seq_len_q, d_head]`, `k`/`v`: `[seq_len_k, d_head]`, `out`:
/// `[seq_len_q, d_head]`, row-major.  Scale `1/sqrt(d_head)`; with `causal`,
/// query `i` sees keys `j <= i`.
///
/// # Panics
///
/// If any slice length differs from its shape.
#[allow(clippy::too_many_arguments)]
pub fn naive_attention(q: &[f32], k: &[f32], v: &[f32], seq_len_q: usize, seq_len_k: usize,
                       d_head: usize, causal: bool, out: &mut [f32]) {
    assert_eq!(q.len(), seq_len_q * d_head);
    assert_eq!(k.len(), seq_len_k * d_head);
    assert_eq!(v.len(), seq_len_k * d_head);
    assert_eq!(out.len(), seq_len_q * d_head);
    let scale = 1.0 / (d_head as f32).sqrt();
    let mut p = vec![0.0f32; seq_len_k];
    for i in 0..seq_len_q {
        let qi = &q[i * d_head..(i + 1) * d_head];
        let mut m = f32::NEG_INFINITY;
        for (j, pj) in p.iter_mut().enumerate() {
            if causal && j > i {
                *pj = f32::NEG_INFINITY;
                continue;
            }
            let kj = &k[j * d_head..(j + 1) * d_head];
            let dot: f32 = qi.iter().zip(kj).map(|(a, b)| a * b).sum();
            *pj = dot * scale;
            m = m.max(*pj);
        }
        let mut sum = 0.0f32;
        for pj in p.iter_mut() {
            *pj = (*pj - m).exp();
            sum += *pj;
        }
        let inv = if sum > 0.0 { 1.0 / sum } else { 0.0 };
        let o = &mut out[i * d_head..(i + 1) * d_head];
        o.fill(0.0);
        for (j, &pj) in p.iter().enumerate() {
            let w = pj * inv;
            if w == 0.0 {
                continue;
            }
            for (oc, vc) in o.iter_mut().zip(&v[j * d_head..(j + 1) * d_head]) {
                *oc += w * vc;
            }
        }
    }
}
