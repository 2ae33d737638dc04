//! Tensor-parallel routed-MoE group: one persistent thread per rank, one B200
//! per thread, the fp32 partials summed by the peer-memory finish.
//!
//! This is the execution boundary the reference's `Tp4WorkerPool` /
//! `RankExecutor::execute` (`crates/glm-engine/src/worker.rs:37-52,595-660`)
//! drives, generalised to 1/2/4/8 ranks: every rank thread owns its context,
//! weights and buffers (thread-affine, as the reference requires); a step
//! broadcasts the input rows, each rank runs `glmaxx_moe_layer_launch` into its
//! partial, and every rank then launches `glmaxx_moe_finish_peer_launch` at the
//! same point of its stream, which adds the partials in rank order
//! (`finish_sparse_layer_oracle`, `crates/glm-reference/src/routed_fc2.rs:214-258`)
//! in place of the NCCL all-reduce of `crates/glm-engine/src/manifest.rs:228`.
//! The result is the same bits on every rank.

use core::ffi::c_void;
use std::sync::mpsc;
use std::sync::{Arc, Barrier, Mutex};
use std::thread::JoinHandle;

use crate::abi::{self, check, KernelError, MoeFinishDescriptor, MoePeerDescriptor};
use crate::ffi;
use crate::rank::{DeviceBuffer, LayerGeometry, RankContext, RankLayerWeights, RoutedMoeStep};

enum Command {
    Step { tokens: u32, input: Arc<Vec<u16>> },
    Shutdown,
}

/// One rank's answer to a step: the finished fp32 rows `[tokens][hidden]`.
pub struct StepOutput {
    pub rank: u32,
    pub output: Vec<f32>,
}

/// Per-rank device addresses every rank needs for the peer finish.
#[derive(Clone, Copy, Default)]
struct RankBuffers {
    partial: u64,
    out: u64,
    signal: u64,
}

pub struct TpMoeGroup {
    ranks: u32,
    hidden: u32,
    commands: Vec<mpsc::Sender<Command>>,
    results: mpsc::Receiver<(u32, Result<StepOutput, KernelError>)>,
    threads: Vec<JoinHandle<()>>,
}

impl TpMoeGroup {
    /// Spawns `ranks` rank threads.  `load(ctx)` runs on each rank's thread after
    /// the device is bound and returns the addresses of that rank's layer shards
    /// (loaded, for example, from its `.g5n` rank file with
    /// `glmaxx_rank_file_verify_and_stream`).
    pub fn spawn<F>(ranks: u32, geometry: LayerGeometry, max_tokens: u32, load: F) -> Result<Self, KernelError>
    where
        F: Fn(&RankContext) -> Result<RankLayerWeights, KernelError> + Send + Sync + 'static,
    {
        if !matches!(ranks, 1 | 2 | 4 | 8) {
            return Err(KernelError::Topology);
        }
        let load = Arc::new(load);
        let table = Arc::new(Mutex::new(vec![RankBuffers::default(); ranks as usize]));
        let ready = Arc::new(Barrier::new(ranks as usize + 1));
        let setup_errors = Arc::new(Mutex::new(Vec::<KernelError>::new()));
        let (result_tx, results) = mpsc::channel();
        let mut commands = Vec::new();
        let mut threads = Vec::new();
        for rank in 0..ranks {
            let (tx, rx) = mpsc::channel::<Command>();
            commands.push(tx);
            let (load, table, ready, errors, results) =
                (load.clone(), table.clone(), ready.clone(), setup_errors.clone(), result_tx.clone());
            threads.push(std::thread::spawn(move || {
                rank_thread(rank, ranks, geometry, max_tokens, &*load, &table, &ready, &errors, &rx, &results);
            }));
        }
        ready.wait(); // every rank bound, loaded and published its buffers
        if let Some(e) = setup_errors.lock().map_err(|_| KernelError::Topology)?.first().copied() {
            for c in &commands {
                let _ = c.send(Command::Shutdown);
            }
            return Err(e);
        }
        Ok(Self { ranks, hidden: geometry.hidden, commands, results, threads })
    }

    /// One layer step over `tokens` bf16 rows (`input.len() == tokens * hidden`):
    /// returns rank 0's finished rows (every rank holds the same bits).
    pub fn step(&self, tokens: u32, input: Vec<u16>) -> Result<Vec<f32>, KernelError> {
        if input.len() != tokens as usize * self.hidden as usize {
            return Err(KernelError::Descriptor);
        }
        let input = Arc::new(input);
        for c in &self.commands {
            c.send(Command::Step { tokens, input: input.clone() }).map_err(|_| KernelError::Topology)?;
        }
        let mut out = None;
        let mut first_err = None;
        for _ in 0..self.ranks {
            let (_, r) = self.results.recv().map_err(|_| KernelError::Topology)?;
            match r {
                Ok(o) if o.rank == 0 => out = Some(o.output),
                Ok(_) => {}
                Err(e) => first_err = first_err.or(Some(e)),
            }
        }
        match first_err {
            Some(e) => Err(e),
            None => out.ok_or(KernelError::Topology),
        }
    }
}

impl Drop for TpMoeGroup {
    fn drop(&mut self) {
        for c in &self.commands {
            let _ = c.send(Command::Shutdown);
        }
        for t in self.threads.drain(..) {
            let _ = t.join();
        }
    }
}

#[allow(clippy::too_many_arguments)]
fn rank_thread(
    rank: u32,
    ranks: u32,
    geometry: LayerGeometry,
    max_tokens: u32,
    load: &(dyn Fn(&RankContext) -> Result<RankLayerWeights, KernelError> + Send + Sync),
    table: &Mutex<Vec<RankBuffers>>,
    ready: &Barrier,
    errors: &Mutex<Vec<KernelError>>,
    commands: &mpsc::Receiver<Command>,
    results: &mpsc::Sender<(u32, Result<StepOutput, KernelError>)>,
) {
    let setup = (|| -> Result<_, KernelError> {
        let ctx = RankContext::bind(rank, ranks)?;
        let weights = load(&ctx)?;
        let step = RoutedMoeStep::new(&ctx, geometry, weights, max_tokens)?;
        let rows = u64::from(max_tokens) * u64::from(geometry.hidden);
        let input = DeviceBuffer::alloc(rows * 2)?;
        let partial = DeviceBuffer::alloc(rows * 4)?;
        let out = DeviceBuffer::alloc(rows * 4)?;
        // SAFETY: pure size query.
        let signal_bytes = unsafe { ffi::glmaxx_moe_peer_signal_bytes(ranks) };
        let signal = DeviceBuffer::zeroed(signal_bytes, ctx.stream()?)?;
        for peer in 0..ranks {
            if peer != rank {
                // SAFETY: enables this device's access to a peer's memory (idempotent).
                check(unsafe { ffi::glmaxx_peer_enable(peer as i32) })?;
            }
        }
        ctx.synchronize()?;
        table.lock().map_err(|_| KernelError::Topology)?[rank as usize] =
            RankBuffers { partial: partial.ptr, out: out.ptr, signal: signal.ptr };
        Ok((ctx, step, input, partial, out, signal))
    })();
    let state = match setup {
        Ok(s) => Some(s),
        Err(e) => {
            if let Ok(mut v) = errors.lock() {
                v.push(e);
            }
            None
        }
    };
    ready.wait();
    let Some((ctx, step, input, _partial, out, _signal)) = state else { return };
    let peers = match table.lock() {
        Ok(t) => t.clone(),
        Err(_) => return,
    };
    while let Ok(cmd) = commands.recv() {
        let Command::Step { tokens, input: rows } = cmd else { break };
        let r = run_step(&ctx, &step, &input, &peers, rank, ranks, tokens, &rows, out.ptr);
        if results.send((rank, r)).is_err() {
            break;
        }
    }
}

#[allow(clippy::too_many_arguments)]
fn run_step(
    ctx: &RankContext,
    step: &RoutedMoeStep,
    input: &DeviceBuffer,
    peers: &[RankBuffers],
    rank: u32,
    ranks: u32,
    tokens: u32,
    rows: &[u16],
    out: u64,
) -> Result<StepOutput, KernelError> {
    let stream = ctx.stream()?;
    let elements = u64::from(tokens) * u64::from(step.geometry.hidden);
    // SAFETY: `rows` holds `elements` bf16 values; `input` has room for max_tokens rows.
    check(unsafe { ffi::glmaxx_memcpy_h2d(input.ptr, rows.as_ptr().cast(), elements * 2, stream) })?;
    let me = peers[rank as usize];
    step.launch(ctx, tokens, input.ptr, me.partial)?;
    // the peer finish: every rank's partial in rank order into this rank's output
    let partials: Vec<u64> = peers.iter().map(|p| p.partial).collect();
    let signals: Vec<u64> = peers.iter().map(|p| p.signal).collect();
    let outs: Vec<u64> = peers.iter().map(|p| p.out).collect();
    let mut fin = MoeFinishDescriptor::new();
    fin.ranks = ranks;
    fin.elements = elements;
    fin.partials_f32 = partials.as_ptr() as u64;
    fin.output_f32 = out;
    // two-shot from 1 MB on with more than two ranks, from 8 MB on with two
    // (the measured crossover of the Python host, glmaxx_b200/peer.py two_shot_pays)
    let bytes = elements * 4;
    let two_shot = if ranks == 2 { bytes >= 8 << 20 } else { ranks > 2 && bytes >= 1 << 20 };
    let mut peer = MoePeerDescriptor::new();
    peer.flags = if two_shot { abi::MOE_PEER_TWO_SHOT } else { abi::MOE_PEER_ONE_SHOT };
    peer.rank = rank;
    peer.signals_u32 = signals.as_ptr() as u64;
    peer.outputs_f32 = if two_shot { outs.as_ptr() as u64 } else { 0 };
    // SAFETY: the descriptors and the host arrays they name live until the call
    // returns (the library reads them at launch); device buffers outlive the step.
    check(unsafe { ffi::glmaxx_moe_finish_peer_launch(&fin, &peer, stream as *mut c_void) })?;
    let mut output = vec![0_f32; elements as usize];
    // SAFETY: `output` has room for `elements` floats.
    check(unsafe { ffi::glmaxx_memcpy_d2h(output.as_mut_ptr().cast(), out, elements * 4, stream) })?;
    step.device_status(ctx)?; // synchronises the stream and checks the status word
    Ok(StepOutput { rank, output })
}
