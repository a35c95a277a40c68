//! The `b200` module of the vestra-kernels crate: the crate's public
//! specialised functions (src/lib.rs:52-130) with the same names, argument
//! order and `bool` results, running on a B200 through libvestra_b200.so.
//! `B200` owns one context (one GPU, one stream), as `CudaRuntime` does
//! (src/cuda.rs:356-388).  Not compiled in this repository (no Rust
//! toolchain here).
pub mod ffi;

use cudarc::driver::{CudaContext, CudaSlice, CudaStream, DevicePtr, DevicePtrMut};
use std::sync::Arc;

pub struct B200 {
    ctx: *mut ffi::VkCtx,
    stream: Arc<CudaStream>,
}

#[derive(Debug)]
pub struct B200Error(pub i32, pub String);

fn last_error() -> String {
    unsafe { std::ffi::CStr::from_ptr(ffi::vk_last_error()) }.to_string_lossy().into_owned()
}

/// VK_OK -> Ok(true); VK_UNSUPPORTED_SHAPE -> Ok(false), the reference's
/// `false` with the output untouched; anything else -> Err.
fn status(code: i32) -> Result<bool, B200Error> {
    match code {
        ffi::VK_OK => Ok(true),
        ffi::VK_UNSUPPORTED_SHAPE => Ok(false),
        c => Err(B200Error(c, last_error())),
    }
}

impl B200 {
    pub fn new(device: usize) -> Result<Self, B200Error> {
        let cu = CudaContext::new(device).map_err(|e| B200Error(ffi::VK_ERR_CUDA, e.to_string()))?;
        let stream = cu.new_stream().map_err(|e| B200Error(ffi::VK_ERR_CUDA, e.to_string()))?;
        let mut ctx = std::ptr::null_mut();
        status(unsafe { ffi::vk_init(device as i32, &mut ctx) })?;
        status(unsafe { ffi::vk_stream_set(ctx, stream.cu_stream() as *mut _) })?;
        Ok(Self { ctx, stream })
    }

    /// VK_MATH_F32 (bit-identical to the reference's projections),
    /// VK_MATH_BF16 or VK_MATH_Q8_0.
    pub fn set_math(&self, math: i32) -> Result<(), B200Error> {
        status(unsafe { ffi::vk_set_math(self.ctx, math) }).map(|_| ())
    }

    fn upload(&self, x: &[f32]) -> CudaSlice<f32> {
        self.stream.memcpy_stod(x).expect("host to device copy")
    }

    /// Runs `call` on device copies of `inputs` and an output of `out.len()`
    /// values; copies the output back only when the call returned VK_OK.
    fn run<F>(&self, inputs: &[&[f32]], out: &mut [f32], call: F) -> bool
    where
        F: FnOnce(&[*const f32], *mut f32) -> i32,
    {
        let s = &self.stream;
        let dev: Vec<CudaSlice<f32>> = inputs.iter().map(|x| self.upload(x)).collect();
        let mut o: CudaSlice<f32> = s.alloc_zeros(out.len()).expect("device output");
        let ok = {
            let guards: Vec<_> = dev.iter().map(|d| d.device_ptr(s)).collect();
            let ptrs: Vec<*const f32> = guards.iter().map(|(p, _)| *p as *const f32).collect();
            let (po, _go) = o.device_ptr_mut(s);
            status(call(&ptrs, po as *mut f32))
        };
        match ok {
            Ok(true) => {
                s.memcpy_dtoh(&o, out).expect("device to host copy");
                true
            }
            _ => false,
        }
    }

    /// qkv_f32_da3_base (src/lib.rs:52): input [tokens, 768], weight
    /// [768, 2304], bias [2304] -> q, k, v [12, tokens, 64].
    pub fn qkv_f32_da3_base(&self, input: &[f32], weight: &[f32], bias: &[f32], q: &mut [f32], k: &mut [f32],
                            v: &mut [f32]) -> bool {
        if input.len() % 768 != 0 || weight.len() != 768 * 2304 || bias.len() != 2304 {
            return false;
        }
        let tokens = input.len() / 768;
        if q.len() != tokens * 768 || k.len() != q.len() || v.len() != q.len() {
            return false;
        }
        let mut qkv = vec![0.0f32; 3 * q.len()];
        let n = q.len();
        let ok = self.run(&[input, weight, bias], &mut qkv, |p, o| unsafe {
            ffi::vk_qkv_f32_da3_base(self.ctx, tokens, p[0], p[1], p[2], o, o.add(n), o.add(2 * n))
        });
        if ok {
            q.copy_from_slice(&qkv[..n]);
            k.copy_from_slice(&qkv[n..2 * n]);
            v.copy_from_slice(&qkv[2 * n..]);
        }
        ok
    }

    /// linear_f32_da3_base (src/lib.rs:67).
    pub fn linear_f32_da3_base(&self, m: usize, n: usize, k: usize, input: &[f32], weight: &[f32],
                               output: &mut [f32]) -> bool {
        if input.len() != m * k || weight.len() != k * n || output.len() != m * n {
            return false;
        }
        self.run(&[input, weight], output, |p, o| unsafe {
            ffi::vk_linear_f32_da3_base(self.ctx, m, n, k, p[0], p[1], o)
        })
    }

    /// flash_attention_f32_da3_base (src/lib.rs:82): q, k, v, out
    /// [heads, tokens, 64].
    pub fn flash_attention_f32_da3_base(&self, q: &[f32], k: &[f32], v: &[f32], heads: usize, tokens: usize,
                                        out: &mut [f32]) -> bool {
        let n = heads * tokens * 64;
        if q.len() != n || k.len() != n || v.len() != n || out.len() != n {
            return false;
        }
        self.run(&[q, k, v], out, |p, o| unsafe {
            ffi::vk_flash_attention_f32_da3_base(self.ctx, p[0], p[1], p[2], heads, tokens, o)
        })
    }

    /// linear_bias_scale_f32_da3_base (src/lib.rs:94): (a b + bias) * scale.
    pub fn linear_bias_scale_f32_da3_base(&self, m: usize, n: usize, k: usize, a: &[f32], b: &[f32],
                                          bias: &[f32], scale: &[f32], c: &mut [f32]) -> bool {
        if a.len() != m * k || b.len() != k * n || bias.len() != n || scale.len() != n || c.len() != m * n {
            return false;
        }
        self.run(&[a, b, bias, scale], c, |p, o| unsafe {
            ffi::vk_linear_bias_scale_f32_da3_base(self.ctx, m, n, k, p[0], p[1], p[2], p[3], o)
        })
    }

    /// qk_norm_rope_f32_da3_base (src/lib.rs:108): q and k [12, tokens, 64]
    /// in place; positions [tokens, 2] (y, x).
    #[allow(clippy::too_many_arguments)]
    pub fn qk_norm_rope_f32_da3_base(&self, q: &mut [f32], k: &mut [f32], q_gamma: &[f32], q_beta: &[f32],
                                     k_gamma: &[f32], k_beta: &[f32], positions_yx: &[i64], frequency: f32,
                                     epsilon: f32) -> bool {
        if q.len() % (12 * 64) != 0 || k.len() != q.len() {
            return false;
        }
        let tokens = q.len() / (12 * 64);
        if positions_yx.len() != 2 * tokens || q_gamma.len() != 64 || q_beta.len() != 64 || k_gamma.len() != 64
            || k_beta.len() != 64 {
            return false;
        }
        let s = &self.stream;
        let mut dq = self.upload(q);
        let mut dk = self.upload(k);
        let (g0, b0, g1, b1) = (self.upload(q_gamma), self.upload(q_beta), self.upload(k_gamma), self.upload(k_beta));
        let dp = s.memcpy_stod(positions_yx).expect("positions");
        let ok = {
            let (pq, _a) = dq.device_ptr_mut(s);
            let (pk, _b) = dk.device_ptr_mut(s);
            let (pg0, _c) = g0.device_ptr(s);
            let (pb0, _d) = b0.device_ptr(s);
            let (pg1, _e) = g1.device_ptr(s);
            let (pb1, _f) = b1.device_ptr(s);
            let (pp, _g) = dp.device_ptr(s);
            status(unsafe {
                ffi::vk_qk_norm_rope_f32_da3_base(self.ctx, pq as *mut f32, pk as *mut f32, 12, tokens,
                                                  pg0 as *const f32, pb0 as *const f32, pg1 as *const f32,
                                                  pb1 as *const f32, pp as *const i64, frequency, epsilon)
            })
        };
        match ok {
            Ok(true) => {
                s.memcpy_dtoh(&dq, q).expect("q back");
                s.memcpy_dtoh(&dk, k).expect("k back");
                true
            }
            _ => false,
        }
    }
}

impl Drop for B200 {
    fn drop(&mut self) {
        unsafe {
            ffi::vk_destroy(self.ctx);
        }
    }
}
