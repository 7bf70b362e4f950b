//! strata-core's [`ComputeBackend`] on B200 GPUs through `libstrata_cuda`.
//!
//! The quantized matrix-vector products (`gemv`, `expert_gemv`, the
//! `crates/strata-core/src/backend.rs:20-51` seam) run on the device, with
//! weights uploaded once and kept resident in HBM, keyed by their slice of the
//! memory-mapped model (stable for the process lifetime, as
//! `crates/strata-core/src/engine.rs` holds the mapping) and evicted least
//! recently used first under a byte budget, as the wgpu backend's weight cache
//! does (`crates/strata-backend-wgpu/src/gpu.rs:61-112`). The elementwise
//! trait methods run on the device too, with the CPU path's f64 arithmetic.
//!
//! Beyond the trait: [`CudaBackend::gemm`] (a whole prompt through one
//! projection — the bf16-staged tensor-core GEMM), [`CudaBackend::moe_layer`]
//! / [`CudaBackend::moe_ffn`] (route, experts, shared expert and combine in
//! one device call) and [`CudaBackend::preload`] (every tensor resident before
//! the first token, in one staged pass).
//!
//! There is no CPU fallback: a type the device does not take is
//! [`Error::UnsupportedQuant`], any device failure is [`Error::Backend`] with
//! the library's message.

mod ffi;

use std::collections::HashMap;
use std::ffi::CStr;
use std::fmt;
use std::sync::Mutex;

use strata_core::backend::{ComputeBackend, QuantTensor, RopeCfg};
use strata_core::error::{Error, Result};
use strata_core::moe::MoeLayer;
use strata_core::weights::ExpertView;
use strata_gguf::quant::QuantType;

/// Tokens per device GEMV call (the library's batch limit).
const GEMV_MAX_BATCH: usize = 8;

/// The quantized-matmul backend on one CUDA device.
pub struct CudaBackend {
    ctx: *mut ffi::StrataCtx,
    cache: Mutex<Cache>,
}

// The library serialises calls per context; the raw handle is only passed to it.
unsafe impl Send for CudaBackend {}
unsafe impl Sync for CudaBackend {}

#[derive(Debug, Default)]
struct Cache {
    /// (slice address, slice length) -> resident tensor
    entries: HashMap<(usize, usize), Entry>,
    bytes: u64,
    budget: u64,
    clock: u64,
}

#[derive(Debug, Clone, Copy)]
struct Entry {
    weight: usize, // *mut ffi::StrataWeight
    bytes: u64,
    last_use: u64,
}

impl fmt::Debug for CudaBackend {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        let c = self.cache.lock().unwrap();
        f.debug_struct("CudaBackend")
            .field("resident_tensors", &c.entries.len())
            .field("resident_bytes", &c.bytes)
            .field("budget", &c.budget)
            .finish()
    }
}

/// A device MoE layer made by [`CudaBackend::moe_layer`].
#[derive(Debug)]
pub struct CudaMoe {
    layer: *mut ffi::StrataMoe,
    n_embd: usize,
    n_expert: usize,
    top_k: usize,
}

unsafe impl Send for CudaMoe {}
unsafe impl Sync for CudaMoe {}

impl Drop for CudaMoe {
    fn drop(&mut self) {
        unsafe {
            ffi::strata_cuda_moe_destroy(self.layer);
        }
    }
}

/// Whether the bf16-staged prefill GEMM takes this matrix; other matrices go
/// through device GEMVs of up to eight tokens each.
fn gemm_takes(quant: QuantType, cols: usize) -> bool {
    matches!(quant, QuantType::Q4K | QuantType::Q5K | QuantType::Q6K) && cols % 256 == 0
}

impl CudaBackend {
    /// A context on `device` whose resident weights may take up to
    /// `budget_bytes` of HBM (least recently used evicted first).
    pub fn new(device: i32, budget_bytes: u64) -> Result<Self> {
        let abi = unsafe { ffi::strata_cuda_abi_version() };
        if abi != ffi::STRATA_CUDA_ABI_VERSION {
            return Err(Error::Backend {
                message: format!("libstrata_cuda ABI {abi}, this crate binds {}", ffi::STRATA_CUDA_ABI_VERSION),
            });
        }
        let mut ctx = std::ptr::null_mut();
        let rc = unsafe { ffi::strata_cuda_create(device, &mut ctx) };
        if rc != ffi::STRATA_OK {
            return Err(Error::Backend {
                message: format!("cuda device {device}: strata_cuda_create returned {rc}"),
            });
        }
        let cache = Cache {
            budget: budget_bytes,
            ..Cache::default()
        };
        Ok(Self {
            ctx,
            cache: Mutex::new(cache),
        })
    }

    fn last_error(&self) -> String {
        let msg = unsafe { CStr::from_ptr(ffi::strata_cuda_last_error(self.ctx)) };
        msg.to_string_lossy().into_owned()
    }

    fn check(&self, rc: i32, quant: QuantType) -> Result<()> {
        match rc {
            ffi::STRATA_OK => Ok(()),
            ffi::STRATA_ERR_UNSUPPORTED_QUANT => Err(Error::UnsupportedQuant {
                quant: quant.to_string(),
            }),
            _ => Err(Error::Backend {
                message: self.last_error(),
            }),
        }
    }

    /// The resident copy of a tensor, uploaded on first use.
    fn resident(&self, data: &[u8], quant: QuantType, n_expert: usize, rows: usize, cols: usize)
        -> Result<*const ffi::StrataWeight> {
        let key = (data.as_ptr() as usize, data.len());
        let mut c = self.cache.lock().unwrap();
        c.clock += 1;
        let now = c.clock;
        if let Some(e) = c.entries.get_mut(&key) {
            e.last_use = now;
            return Ok(e.weight as *const ffi::StrataWeight);
        }
        let bytes = data.len() as u64;
        while !c.entries.is_empty() && c.bytes + bytes > c.budget {
            let victim = *c.entries.iter().min_by_key(|(_, e)| e.last_use).map(|(k, _)| k).unwrap();
            let e = c.entries.remove(&victim).unwrap();
            c.bytes -= e.bytes;
            unsafe {
                ffi::strata_cuda_free_weight(e.weight as *mut ffi::StrataWeight);
            }
        }
        let mut w = std::ptr::null_mut();
        let rc = unsafe {
            ffi::strata_cuda_upload(
                self.ctx,
                data.as_ptr(),
                data.len(),
                quant.id(),
                n_expert as i64,
                rows as i64,
                cols as i64,
                &mut w,
            )
        };
        self.check(rc, quant)?;
        c.entries.insert(
            key,
            Entry {
                weight: w as usize,
                bytes,
                last_use: now,
            },
        );
        c.bytes += bytes;
        Ok(w)
    }

    fn dense(&self, w: &QuantTensor<'_>) -> Result<*const ffi::StrataWeight> {
        self.resident(w.data, w.quant, 0, w.rows, w.cols)
    }

    fn experts(&self, w: &ExpertView<'_>) -> Result<*const ffi::StrataWeight> {
        self.resident(w.data, w.quant, w.n_expert, w.rows, w.cols)
    }

    /// `ys[t] = W xs[t]` for every token `t` of a prompt (`xs` holds
    /// `xs.len() / w.cols` rows): one tensor-core GEMM on the bf16-rounded
    /// activations (within 1e-2 of `ops::gemv` on the rounded input) where
    /// the format allows, else device GEMVs of up to eight tokens each.
    pub fn gemm(&self, w: &QuantTensor<'_>, xs: &[f32], ys: &mut [f32]) -> Result<()> {
        let m = xs.len() / w.cols;
        assert!(ys.len() >= m * w.rows, "gemm: output holds fewer than {m} rows of {}", w.rows);
        if m == 0 {
            return Ok(());
        }
        let dw = self.dense(w)?;
        if gemm_takes(w.quant, w.cols) {
            let rc = unsafe { ffi::strata_cuda_gemm_f32(self.ctx, dw, xs.as_ptr(), ys.as_mut_ptr(), m as i64) };
            return self.check(rc, w.quant);
        }
        self.gemv_loop(dw, w, xs, ys, m)
    }

    fn gemv_loop(&self, dw: *const ffi::StrataWeight, w: &QuantTensor<'_>, xs: &[f32], ys: &mut [f32], m: usize)
        -> Result<()> {
        let mut t = 0;
        while t < m {
            let b = (m - t).min(GEMV_MAX_BATCH);
            let x = xs[t * w.cols..(t + b) * w.cols].as_ptr();
            let y = ys[t * w.rows..(t + b) * w.rows].as_mut_ptr();
            let rc = unsafe { ffi::strata_cuda_gemv(self.ctx, dw, x, y, b as i32) };
            self.check(rc, w.quant)?;
            t += b;
        }
        Ok(())
    }

    /// The device MoE layer for `layer` (`crates/strata-core/src/moe.rs`):
    /// router, all experts and the shared expert, resident. Under expert
    /// parallelism a rank passes its expert range and whether it runs the
    /// shared expert; one process holding the whole layer passes
    /// `0..layer.n_expert` and `true`.
    pub fn moe_layer(&self, layer: &MoeLayer<'_>, experts: std::ops::Range<usize>, with_shared: bool)
        -> Result<CudaMoe> {
        let n_embd = layer.router.cols;
        let desc = ffi::strata_moe_desc {
            router: self.dense(&layer.router)?,
            gate_exps: self.experts(&layer.gate_exps)?,
            up_exps: self.experts(&layer.up_exps)?,
            down_exps: self.experts(&layer.down_exps)?,
            gate_shexp: self.dense(&layer.gate_shexp)?,
            up_shexp: self.dense(&layer.up_shexp)?,
            down_shexp: self.dense(&layer.down_shexp)?,
            gate_inp_shexp: self.dense(&layer.gate_inp_shexp)?,
            n_embd: n_embd as i64,
            n_expert: layer.n_expert as i64,
            top_k: layer.top_k as i64,
            n_ff: layer.n_ff as i64,
            n_ff_shexp: layer.gate_shexp.rows as i64,
            expert_begin: experts.start as i64,
            expert_end: experts.end as i64,
            with_shared: i32::from(with_shared),
        };
        let mut out = std::ptr::null_mut();
        let rc = unsafe { ffi::strata_cuda_moe_create(self.ctx, &desc, &mut out) };
        self.check(rc, layer.gate_exps.quant)?;
        Ok(CudaMoe {
            layer: out,
            n_embd,
            n_expert: layer.n_expert,
            top_k: layer.top_k,
        })
    }

    /// The MoE half for `xs.len() / n_embd` tokens, as `MoeLayer::forward`
    /// computes it: routing from the router GEMV on the bf16-rounded input
    /// (softmax over all experts, top-k with ties to the lower index,
    /// renormalised), the routed experts, the sigmoid-gated shared expert,
    /// the combine. `routing`, when given, receives each token's expert ids
    /// and weights (`top_k` of each per token).
    pub fn moe_ffn(&self, moe: &CudaMoe, xs: &[f32], out: &mut [f32], routing: Option<(&mut [i32], &mut [f32])>)
        -> Result<()> {
        let tokens = xs.len() / moe.n_embd;
        assert!(out.len() >= tokens * moe.n_embd, "moe_ffn: output holds fewer than {tokens} tokens");
        let (ids, wts) = match routing {
            Some((ids, wts)) => {
                assert!(ids.len() >= tokens * moe.top_k && wts.len() >= tokens * moe.top_k);
                (ids.as_mut_ptr(), wts.as_mut_ptr())
            }
            None => (std::ptr::null_mut(), std::ptr::null_mut()),
        };
        let rc = unsafe {
            ffi::strata_cuda_moe_ffn(
                self.ctx,
                moe.layer,
                xs.as_ptr(),
                std::ptr::null(),
                tokens as i64,
                out.as_mut_ptr(),
                ids,
                wts,
            )
        };
        if rc == ffi::STRATA_OK {
            Ok(())
        } else {
            Err(Error::Backend {
                message: format!("moe ffn ({} experts): {}", moe.n_expert, self.last_error()),
            })
        }
    }

    /// Every matrix and expert tensor of the model resident before the first
    /// token, in one staged pass (two pinned chunks, host threads taking the
    /// mapping's page faults while the copy engine drains the other chunk).
    /// All or nothing: on an error no tensor of the call stays resident.
    pub fn preload(&self, views: &[QuantTensor<'_>], experts: &[ExpertView<'_>]) -> Result<()> {
        let mut items = Vec::with_capacity(views.len() + experts.len());
        let mut keys = Vec::with_capacity(items.capacity());
        for v in views {
            items.push(ffi::strata_upload {
                bytes: v.data.as_ptr(),
                len: v.data.len(),
                quant: v.quant.id(),
                n_expert: 0,
                rows: v.rows as i64,
                cols: v.cols as i64,
            });
            keys.push((v.data.as_ptr() as usize, v.data.len()));
        }
        for v in experts {
            items.push(ffi::strata_upload {
                bytes: v.data.as_ptr(),
                len: v.data.len(),
                quant: v.quant.id(),
                n_expert: v.n_expert as i64,
                rows: v.rows as i64,
                cols: v.cols as i64,
            });
            keys.push((v.data.as_ptr() as usize, v.data.len()));
        }
        let mut out = vec![std::ptr::null_mut(); items.len()];
        let rc = unsafe { ffi::strata_cuda_upload_many(self.ctx, items.as_ptr(), items.len() as i64, out.as_mut_ptr()) };
        if rc != ffi::STRATA_OK {
            return Err(Error::Backend {
                message: self.last_error(),
            });
        }
        let mut c = self.cache.lock().unwrap();
        for (k, w) in keys.into_iter().zip(out) {
            c.clock += 1;
            let now = c.clock;
            if let Some(old) = c.entries.insert(
                k,
                Entry {
                    weight: w as usize,
                    bytes: k.1 as u64,
                    last_use: now,
                },
            ) {
                c.bytes -= old.bytes;
                unsafe {
                    ffi::strata_cuda_free_weight(old.weight as *mut ffi::StrataWeight);
                }
            }
            c.bytes += k.1 as u64;
        }
        Ok(())
    }
}

impl ComputeBackend for CudaBackend {
    fn name(&self) -> &'static str {
        "cuda"
    }

    fn gemv(&self, w: &QuantTensor<'_>, x: &[f32], y: &mut [f32], _scratch: &mut [f32]) -> Result<()> {
        assert!(x.len() >= w.cols && y.len() >= w.rows, "gemv {}: x or y too short", w.name);
        let dw = self.dense(w)?;
        let rc = unsafe { ffi::strata_cuda_gemv(self.ctx, dw, x.as_ptr(), y.as_mut_ptr(), 1) };
        self.check(rc, w.quant)
    }

    fn expert_gemv(&self, w: &ExpertView<'_>, e: usize, x: &[f32], y: &mut [f32], _scratch: &mut [f32])
        -> Result<()> {
        assert!(x.len() >= w.rows && y.len() >= w.cols, "expert_gemv {}: x or y too short", w.name);
        let dw = self.experts(w)?;
        let rc = unsafe { ffi::strata_cuda_expert_gemv(self.ctx, dw, e as i64, x.as_ptr(), y.as_mut_ptr(), 1) };
        self.check(rc, w.quant)
    }

    fn rms_norm(&self, x: &mut [f32], w: &[f32], eps: f64) -> Result<()> {
        // ops::rms_norm indexes w by the position in x
        assert!(w.len() >= x.len(), "rms_norm: fewer weights than values");
        let rc = unsafe { ffi::strata_cuda_rms_norm(self.ctx, x.as_mut_ptr(), w.as_ptr(), x.len() as i64, eps) };
        self.check(rc, QuantType::F32)
    }

    fn rope_neox(&self, head: &mut [f32], cfg: &RopeCfg) -> Result<()> {
        let rc = unsafe {
            ffi::strata_cuda_rope_neox(
                self.ctx,
                head.as_mut_ptr(),
                head.len() as i64,
                cfg.pos as i64,
                cfg.n_rot as i64,
                cfg.head_dim as i64,
                cfg.freq_base,
            )
        };
        self.check(rc, QuantType::F32)
    }

    fn softmax(&self, xs: &mut [f32]) -> Result<()> {
        let rc = unsafe { ffi::strata_cuda_softmax(self.ctx, xs.as_mut_ptr(), xs.len() as i64) };
        self.check(rc, QuantType::F32)
    }

    fn l2_norm(&self, head: &mut [f32], eps: f64) -> Result<()> {
        let rc = unsafe { ffi::strata_cuda_l2_norm(self.ctx, head.as_mut_ptr(), head.len() as i64, eps) };
        self.check(rc, QuantType::F32)
    }

    fn add(&self, a: &mut [f32], b: &[f32]) -> Result<()> {
        // ops::add_into zips the two slices
        let n = a.len().min(b.len());
        if n == 0 {
            return Ok(());
        }
        let rc = unsafe { ffi::strata_cuda_add(self.ctx, a.as_mut_ptr(), b.as_ptr(), n as i64) };
        self.check(rc, QuantType::F32)
    }
}

impl Drop for CudaBackend {
    fn drop(&mut self) {
        for (_, e) in self.cache.lock().unwrap().entries.drain() {
            unsafe {
                ffi::strata_cuda_free_weight(e.weight as *mut ffi::StrataWeight);
            }
        }
        unsafe {
            ffi::strata_cuda_destroy(self.ctx);
        }
    }
}
