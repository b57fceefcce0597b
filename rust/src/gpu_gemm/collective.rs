//! Lowering of `MatMul -> Collective(AllGather)` over a column-sharded output
//! to the library's fused replicated GEMM (`mmr_sharded_gemm_bind`).
//!
//! The reference IR names the collective (`CollectiveKind::AllGather`,
//! ir.rs:1140-1154) but rejects it until the spec carries a group size and a
//! partition axis (ir.rs:1773-1779). With those two fields frozen in the spec,
//! a GPU plan expresses a column-sharded MatMul whose result is replicated on
//! every rank as two nodes: rank r's MatMul over B[:, c0:c1] (its column
//! block, `mmr_shard_columns` in 256-column units) and an AllGather of the
//! output along its last axis. This backend binds the pair as ONE handle: the
//! GEMM's epilogue stores every finished tile into each rank's replica over
//! NVLink (peer stores through CUDA IPC mappings), and a bounded completion
//! handshake ends the run, so the AllGather node itself launches nothing.
//! The only host exchange is the bind-time swap of IPC handles, carried by
//! whatever process-group transport the embedding runtime provides.
//!
//! NOT COMPILED HERE (no Rust toolchain in the build image).

use core::ptr;

use super::{ffi, status, GpuGemmError};

/// Bind-time transport between the ranks of one node (a TCP store, MPI, or
/// the runtime's own control plane): every rank contributes `mine` and
/// receives every rank's contribution in rank order.
pub trait PeerExchange {
    fn all_gather(&self, mine: &[u8]) -> Result<Vec<Vec<u8>>, GpuGemmError>;
}

/// A rank's replicated column-sharded GEMM: the handle, and the peer buffers
/// it mapped (released after the handle).
pub struct ReplicatedMatMul {
    handle: *mut ffi::mmr_gemm_handle,
    imported: Vec<(u64, ffi::mmr_ipc_handle)>,
}

fn encode(h: &ffi::mmr_ipc_handle) -> Vec<u8> {
    let mut v = h.bytes.to_vec();
    v.extend_from_slice(&h.offset.to_le_bytes());
    v
}

fn decode(b: &[u8]) -> Result<ffi::mmr_ipc_handle, GpuGemmError> {
    if b.len() != 72 {
        return Err(GpuGemmError::InvalidShape);
    }
    let mut h = ffi::mmr_ipc_handle { bytes: [0; 64], offset: 0 };
    h.bytes.copy_from_slice(&b[..64]);
    h.offset = u64::from_le_bytes(b[64..72].try_into().unwrap());
    Ok(h)
}

impl ReplicatedMatMul {
    /// `whole` describes the full node on this rank's device: the full lhs,
    /// rhs and bias, and this rank's full output replica. `signal` is a
    /// zero-initialised device array of `nranks` u64 on this rank.
    ///
    /// # Safety
    /// The buffers named by `whole` and `signal` must outlive the returned
    /// value and every run of it; all ranks must bind the same node.
    pub unsafe fn bind(
        whole: &ffi::mmr_matmul_desc,
        rank: i32,
        nranks: i32,
        signal: u64,
        exchange: &dyn PeerExchange,
    ) -> Result<Self, GpuGemmError> {
        // Every rank validates the same narrowing the bind will use.
        let mut local = *whole;
        let (mut c0, mut c1, mut off) = (0i64, 0i64, 0u64);
        status(ffi::mmr_shard_local_desc(whole, rank, nranks, &mut local, &mut c0, &mut c1, &mut off))?;
        // Export this rank's replica and signal array; collect everyone's.
        let mut out_h = ffi::mmr_ipc_handle { bytes: [0; 64], offset: 0 };
        let mut sig_h = ffi::mmr_ipc_handle { bytes: [0; 64], offset: 0 };
        status(ffi::mmr_ipc_export(whole.out.address, &mut out_h))?;
        status(ffi::mmr_ipc_export(signal, &mut sig_h))?;
        let mut mine = encode(&out_h);
        mine.extend(encode(&sig_h));
        let everyone = exchange.all_gather(&mine)?;
        if everyone.len() != nranks as usize {
            return Err(GpuGemmError::InvalidShape);
        }
        let mut d = ffi::mmr_sharded_desc {
            local: *whole,
            rank,
            nranks,
            peer_out: [0; 8],
            peer_signal: [0; 8],
            signal,
        };
        let mut me = ReplicatedMatMul { handle: ptr::null_mut(), imported: Vec::new() };
        for (r, blob) in everyone.iter().enumerate() {
            if r == rank as usize {
                d.peer_out[r] = whole.out.address;
                d.peer_signal[r] = signal;
                continue;
            }
            if blob.len() != 144 {
                return Err(GpuGemmError::InvalidShape);
            }
            for (i, part) in [&blob[..72], &blob[72..]].iter().enumerate() {
                let h = decode(part)?;
                let mut addr = 0u64;
                status(ffi::mmr_ipc_import(&h, whole.device_ordinal, &mut addr))?;
                me.imported.push((addr, h));
                if i == 0 { d.peer_out[r] = addr } else { d.peer_signal[r] = addr }
            }
        }
        status(ffi::mmr_sharded_gemm_bind(&d, &mut me.handle))?;
        Ok(me)
    }

    /// One run: this rank's column block, stored into every replica, then the
    /// bounded completion handshake with every peer.
    pub fn run(&mut self) -> Result<(), GpuGemmError> {
        status(unsafe { ffi::mmr_gemm_run(self.handle) })
    }

    /// Completion of every run, including every peer's stores into this
    /// replica (MMR_ERR_TIMEOUT when a peer never ran).
    pub fn quiesce(&mut self, timeout_ns: u64) -> Result<(), GpuGemmError> {
        status(unsafe { ffi::mmr_gemm_quiesce(self.handle, timeout_ns) })
    }
}

impl Drop for ReplicatedMatMul {
    fn drop(&mut self) {
        if !self.handle.is_null() {
            unsafe { ffi::mmr_gemm_destroy(self.handle) };
        }
        for (addr, h) in self.imported.drain(..) {
            unsafe { ffi::mmr_ipc_release(addr, &h) };
        }
    }
}
