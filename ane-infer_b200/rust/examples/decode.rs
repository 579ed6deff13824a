//! Greedy decode timing through the Rust binding, in the shape of the reference CLI's GPU
//! bench (crates/cli/src/main.rs:418-498): one warm-up token, then (n_gen - 1) timed tokens.
//!
//!     cargo run --release --example decode -- model.gguf [n_gen]
use std::time::Instant;

fn main() -> Result<(), Box<dyn std::error::Error>> {
    let mut args = std::env::args().skip(1);
    let path = args.next().ok_or("usage: decode MODEL.gguf [n_gen]")?;
    let n_gen: usize = args.next().map(|s| s.parse()).transpose()?.unwrap_or(128);
    let gguf = std::fs::read(&path)?;
    let cfg = ab2::inspect(&gguf)?;
    eprintln!("  Model: {} layers, dim {}, vocab {}", cfg.n_layers, cfg.dim, cfg.vocab);
    let mut dec = ab2::Decoder::new(&gguf, 0, 1, (n_gen + 2) as i32, &ab2::Options::default())?;
    dec.set_step_graph(true)?;
    let mut tok = 1i32;
    let mut generated = vec![];
    let mut t0 = Instant::now();
    for i in 0..n_gen {
        if i == 1 {
            t0 = Instant::now();
        }
        tok = dec.decode_greedy(&[tok])?[0];
        generated.push(tok);
    }
    let secs = t0.elapsed().as_secs_f64();
    let tps = if n_gen > 1 { (n_gen - 1) as f64 / secs } else { 0.0 };
    eprintln!("  Tokens: {n_gen}");
    eprintln!("  Time: {:.1}ms", secs * 1e3);
    eprintln!("  Speed: {tps:.1} tok/s (B200 tg{n_gen})");
    println!("{generated:?}");
    Ok(())
}
