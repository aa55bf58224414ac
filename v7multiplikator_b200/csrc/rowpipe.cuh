// rowpipe.cuh -- persistent row kernels fed by bulk copies (sm_100).
//
// One CTA per SM, W warps, each warp working through its own rows (warp w of
// CTA b of G takes rows b + G w, then every G W rows, so every CTA holds
// rows b, b + G, b + 2G, ... and the SMs' shares differ by one row at most).  Every warp owns S shared-memory slots;
// one lane starts the copy of a future row into a free slot with a 1-D bulk
// copy (cp.async.bulk: the TMA engine without a tensor map, no multicast)
// that completes on the slot's transaction-counting mbarrier, so the row's
// bytes arrive without one load instruction per element and W * S rows per
// SM are in flight at once, outside the load/store unit's queue (whose
// 4-byte-per-lane requests throttled the register-chunk kernels).  The lanes
// then read the row from shared memory in whatever layout the arithmetic
// needs -- the reference's accumulator chains (lane l: elements l + 32k,
// conflict-free) for the sums of squares, float4 for the elementwise pass --
// and write their outputs with 16-byte stores; the slot is refilled as soon
// as every lane is done with it.  gamma is copied once per CTA.
//
// Shared memory of a CTA: gamma (n floats), then the W * S slots (each NIN
// input rows of n floats), then the W * S + 1 mbarriers (the slots', then
// gamma's).  Waits are bounded (pipeline.cuh): a wait that gives up counts
// itself in g_rowpipe_timeouts, the warp stores nothing more and, before it
// leaves, waits (bounded again) for the copies it still has in flight.
#pragma once
#include <cstdint>

#include "launch.cuh"
#include "pipeline.cuh"

namespace v7g {
namespace {

// Bounded waits of the row pipelines of this compilation unit that gave up.
__device__ unsigned int g_rowpipe_timeouts;

constexpr int kPipeMaxWarps = 16;
// dynamic shared memory a row-pipeline CTA may use (B200: 227 KB per CTA)
constexpr uint32_t kPipeSmemBudget = 220u * 1024u;

__host__ __device__ inline uint32_t pipe_round128(uint32_t v) { return (v + 127u) & ~127u; }

struct PipeLayout {
	uint32_t gamma_bytes; // n * 4, rounded up to 128
	uint32_t row_bytes;   // n * 4
	uint32_t slot_bytes;  // NIN rows, rounded up to 128
	int warps, stages;
	__host__ __device__ uint32_t slots_off() const { return gamma_bytes; }
	__host__ __device__ uint32_t bars_off() const { return gamma_bytes + (uint32_t)(warps * stages) * slot_bytes; }
	__host__ __device__ uint32_t total() const { return bars_off() + (uint32_t)(warps * stages + 1) * 8u; }
};

__host__ __device__ inline PipeLayout pipe_layout(int n, int nin, int warps, int stages)
{
	PipeLayout L;
	L.row_bytes = (uint32_t)n * 4u;
	L.gamma_bytes = pipe_round128(L.row_bytes);
	L.slot_bytes = pipe_round128((uint32_t)nin * L.row_bytes);
	L.warps = warps;
	L.stages = stages;
	return L;
}

// Warps per CTA for rows of n floats with NIN inputs per slot and S slots per
// warp within the budget; 0 when fewer than two warps fit.
inline int pipe_warps(int n, int nin, int stages)
{
	for (int w = kPipeMaxWarps; w >= 2; --w)
		if (pipe_layout(n, nin, w, stages).total() <= kPipeSmemBudget)
			return w;
	return 0;
}

// Warps per CTA for a launch: as many as the budget allows, but no more than
// spread the rows over every SM (a few hundred rows in CTAs of 16 warps
// would leave most SMs idle); 0 when the rows are too long for two warps.
inline int pipe_warps_for(int n, int nin, int stages, int64_t rows, int sm_count)
{
	const int w = pipe_warps(n, nin, stages);
	if (w == 0)
		return 0;
	const int64_t spread = (rows + sm_count - 1) / sm_count;
	return (int)(spread < w ? (spread < 1 ? 1 : spread) : w);
}

// One warp's slots.  issue() is called by one lane.
template <int S, int NIN>
struct WarpPipe {
	unsigned char *slot0; // this warp's slot 0
	uint64_t *bar;        // this warp's S barriers
	const float *src[NIN];
	uint32_t slot_bytes, row_bytes;
	int64_t n;
	int64_t issued = 0, waited = 0; // rows started / rows whose wait returned or was abandoned

	__device__ float *slot(int s, int i) const { return reinterpret_cast<float *>(slot0 + (uint32_t)s * slot_bytes + (uint32_t)i * row_bytes); }

	// starts the copy of global row `row` into the slot of the warp's row
	// number `issued` (the copy by the leader lane; every lane counts it)
	__device__ void issue(int64_t row, bool leader)
	{
		const int s = (int)(issued % S);
		if (leader) {
			mbar_arrive_expect_tx(bar + s, NIN * row_bytes);
#pragma unroll
			for (int i = 0; i < NIN; ++i)
				bulk_copy_g2s(slot(s, i), src[i] + row * n, row_bytes, bar + s);
		}
		++issued;
	}

	// waits (all lanes) for the warp's row number `waited`; false when the
	// bound ran out, and then the row stays counted as not waited for, so
	// drain() waits for its copy again
	__device__ bool wait()
	{
		const int64_t k = waited;
		const bool ok = __all_sync(0xffffffffu, mbar_wait(bar + (int)(k % S), (uint32_t)((k / S) & 1), &g_rowpipe_timeouts));
		if (ok)
			++waited;
		return ok;
	}

	// after a failed wait: every copy the warp started and has not seen land
	// (the one whose wait ran out included) lands before the warp leaves, each
	// wait bounded again
	__device__ void drain()
	{
		while (waited < issued) {
			const int64_t k = waited++;
			mbar_wait(bar + (int)(k % S), (uint32_t)((k / S) & 1), &g_rowpipe_timeouts);
		}
	}
};

// CTA set-up shared by the row pipelines: barriers initialised, then (after
// the wait for the kernel ahead in the stream) gamma's copy started.  Returns
// this warp's pipe with its first row started; pipe_wait_gamma starts the
// other S - 1, so that every warp's first row is queued at the copy engine
// before any warp's second.
template <int S, int NIN>
__device__ __forceinline__ WarpPipe<S, NIN> pipe_start(unsigned char *smem, const PipeLayout &L, const float *const (&src)[NIN], const float *w, int64_t n,
                                                      int64_t first_row, int64_t row_step, int64_t rows)
{
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars_off());
	if (threadIdx.x == 0) {
		for (int i = 0; i < L.warps * L.stages + 1; ++i)
			mbar_init(bars + i, 1);
		mbar_init_fence();
	}
	__syncthreads();
	kernel_entry();
	uint64_t *gbar = bars + L.warps * L.stages;
	if (threadIdx.x == 0) {
		mbar_arrive_expect_tx(gbar, L.row_bytes);
		bulk_copy_g2s(smem, w, L.row_bytes, gbar);
	}
	WarpPipe<S, NIN> p;
	p.slot0 = smem + L.slots_off() + (uint32_t)(warp * S) * L.slot_bytes;
	p.bar = bars + warp * S;
#pragma unroll
	for (int i = 0; i < NIN; ++i)
		p.src[i] = src[i];
	p.slot_bytes = L.slot_bytes;
	p.row_bytes = L.row_bytes;
	p.n = n;
	if (first_row < rows)
		p.issue(first_row, lane == 0);
	return p;
}

// Starts the warp's rows 1 .. S-1, then waits (bounded) for gamma's barrier
// (phase 0).  When that wait runs out it waits once more (bounded) before
// returning false, so that gamma's copy, started by the CTA's first thread,
// has landed before any warp of the CTA can leave.
template <int S, int NIN>
__device__ __forceinline__ bool pipe_wait_gamma(WarpPipe<S, NIN> &p, unsigned char *smem, const PipeLayout &L, int64_t first_row, int64_t row_step,
                                                int64_t rows)
{
	const int lane = threadIdx.x & 31;
	for (int s = 1; s < S; ++s) {
		const int64_t row = first_row + s * row_step;
		if (row < rows)
			p.issue(row, lane == 0);
	}
	uint64_t *gbar = reinterpret_cast<uint64_t *>(smem + L.bars_off()) + L.warps * L.stages;
	if (__all_sync(0xffffffffu, mbar_wait(gbar, 0, &g_rowpipe_timeouts)))
		return true;
	mbar_wait(gbar, 0, &g_rowpipe_timeouts);
	return false;
}

// Host: the pipeline kernel's shared-memory ceiling raised to the budget,
// once per device (devices 0..63); `done` is the kernel's own flag word.
template <typename Kernel>
int pipe_allow_smem(Kernel kernel, int device, uint64_t &done)
{
	const uint64_t bit = 1ull << (device & 63);
	if (__atomic_load_n(&done, __ATOMIC_ACQUIRE) & bit)
		return 0;
	if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPipeSmemBudget) != cudaSuccess) {
		cudaGetLastError();
		return -1;
	}
	__atomic_fetch_or(&done, bit, __ATOMIC_ACQ_REL);
	return 0;
}

// Host: this compilation unit's count of given-up pipeline waits.
inline unsigned int rowpipe_timeouts_here()
{
	unsigned int v = 0;
	if (cudaMemcpyFromSymbol(&v, g_rowpipe_timeouts, sizeof(v)) != cudaSuccess) {
		cudaGetLastError();
		return 0xffffffffu;
	}
	return v;
}

} // namespace
} // namespace v7g
