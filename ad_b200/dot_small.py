"""Small dot products on the tcgen05 tensor cores, one kernel per command.

The per-(sequence, head) products of a traced transformer (config 4:
128 x 128 x 64 scores, 128 x 64 x 128 weighted values and their backward
products; 256 of each per layer) are too small for the split + persistent
GEMM path of ``tcgen05.py``: the operands are a few tens of KB, so a
round trip through HBM for the hi/lo split and a deep TMA pipeline cost more
than the product.  Here one CTA computes a 128 x BN tile of one command:

1. all 256 threads gather a K chunk of both operands through their access
   expressions (any folded Permute/View/Broadcast/Concat), split each value
   into ``hi = tf32_rn(x)`` and ``lo = tf32_rn(x - hi)`` in registers, and
   store both into shared memory in the K-major, 64-byte-swizzled layout the
   UMMA descriptors read (the layout a TMA SWIZZLE_64B load would produce);
2. one thread issues ``A_hi*B_hi + A_hi*B_lo + A_lo*B_hi`` per 8-deep K step
   as ``tcgen05.mma.cta_group::1.kind::tf32`` into a TMEM accumulator and
   commits to an mbarrier; the next chunk is gathered after it completes;
3. the 8 warps read the accumulator (``tcgen05.ld.32x32b.x32``), transpose
   32 x 32 blocks through shared memory and run the command's fused epilogue
   with coalesced stores.

The kernel takes only pointer parameters (plus the device error word), so
the batching pass runs the 256 commands of a level as one launch
(``blockIdx.z`` = command).  Every wait is bounded (2 s of ``%globaltimer``);
on expiry the kernel records error code 6, waits (bounded) for the MMAs it
issued, frees its TMEM and returns.

Reference semantics: ``C[ty,tx] = sum_k A(_x=ty,_y=k) * B(_x=k,_y=tx)``
(autodiff/device/opencl/kernels/dotprod.py:7-43) and the epilogue of
dp_elw_fuse.py:11-65, with fp32-level accuracy from the 3xTF32 split.
"""
from __future__ import annotations

from typing import Dict

from . import exprs, ir
from .codegen import KernelSpec, dot_epilogue, dot_shape, index_type, make_emitter, written_reads_bytes

import os

# operand bytes per CTA (hi + lo of A and B for one K chunk): small enough that
# two or three CTAs share an SM, so one CTA's gather overlaps another's MMAs
SMEM_BUDGET = int(os.environ.get("AD_DS_SMEM_KB", "64")) * 1024
SMEM_PER_SM = 228 * 1024
TMEM_COLS = 512


def pad(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def eligible(M: int, N: int, K: int) -> bool:
    """Products this kernel serves well: at least half a 128-row tile, a
    32-column tile and two 8-deep K steps."""
    return M >= 64 and N >= 32 and K >= 16


def tile_shape(N: int, K: int):
    bn = min(256, pad(N, 32))
    kp = pad(K, 16)
    kc = min(kp, (SMEM_BUDGET // ((128 + bn) * 8)) // 16 * 16)
    tcols = 32
    while tcols < bn:
        tcols *= 2
    return bn, kc, tcols


def gen_dot_tc(c, name: str, sizes: Dict[int, int]) -> KernelSpec:
    dn, M, N, K = dot_shape(c)
    BN, KC, TCOLS = tile_shape(N, K)
    NKC = -(-pad(K, 16) // KC)
    rng = {"X": (0, max(M, K) - 1), "Y": (0, max(N, K) - 1), "G": (0, M * N - 1)}
    it = index_type(c, rng)
    bufs, em = make_emitter(c, it)
    A, B = dn.kargs
    la = em.scalar_karg(A, {"X": "gm", "Y": "gk"}, {})
    lb = em.scalar_karg(B, {"X": "gk", "Y": "gn"}, {})
    epi = dot_epilogue(c, em, it, "accv", {"X": "om", "Y": "on", "G": f"(om * ({it}){N} + on)"})
    epi = "\n                    ".join(epi.split("\n"))
    params = ", ".join([f"float* __restrict__ p{i}" for i in range(len(bufs))] + ["int* __restrict__ err"])

    a_load, a_store = _fill(em, A, "A", "Ah", "Al", 128, KC, M, K, "m0", "X", "Y", it)
    b_load, b_store = _fill(em, B, "B", "Bh", "Bl", BN, KC, N, K, "n0", "Y", "X", it)
    A_BYTES, B_BYTES = 128 * KC * 4, BN * KC * 4
    # + alignment slack; the epilogue's 8 x 4 KB transpose buffers reuse the operands
    smem = max(A_BYTES * 2 + B_BYTES * 2, 32 * 1024) + 1024
    # co-resident CTAs must not ask for more TMEM columns than the SM has
    # (2 KB per CTA: static shared memory and the system's reservation)
    if (SMEM_PER_SM // (smem + 2048)) * TCOLS > TMEM_COLS:
        smem = SMEM_PER_SM // (TMEM_COLS // TCOLS) - 2048 + 64
    assert smem <= 225 * 1024
    idesc = (1 << 4) | (2 << 7) | (2 << 10) | ((BN >> 3) << 17) | ((128 >> 4) << 24)
    src = f"""
__device__ __forceinline__ unsigned ds_smem(const void* p) {{ return (unsigned)__cvta_generic_to_shared(p); }}
__device__ __forceinline__ bool ds_try(unsigned long long* b, unsigned ph) {{
    unsigned ok;
    asm volatile("{{\\n .reg .pred p;\\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\\n selp.u32 %0, 1, 0, p;\\n}}"
                 : "=r"(ok) : "r"(ds_smem(b)), "r"(ph) : "memory");
    return ok != 0;
}}
__device__ __noinline__ bool ds_wait(unsigned long long* b, unsigned ph) {{
    if (ds_try(b, ph)) return true;
    unsigned long long t0, t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    while (true) {{
        for (int i = 0; i < 64; ++i) if (ds_try(b, ph)) return true;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (t - t0 > 2000000000ull) return false;
    }}
}}
// K-major operand rows of 16 fp32 (64 bytes) in 8-row swizzle atoms: element (r, k)
// of a K block lands at r * 64 + ((k / 4) ^ ((r / 2) % 4)) * 16 + (k % 4) * 4
__device__ __forceinline__ unsigned ds_off(int r, int k, int rows) {{
    const int kb = k >> 4, kw = k & 15;
    return (unsigned)(kb * rows * 64 + r * 64 + ((((kw >> 2) ^ ((r >> 1) & 3))) << 4) + ((kw & 3) << 2));
}}
__device__ __forceinline__ void ds_split(float x, float& h, float& l) {{
    unsigned hb, lb;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hb) : "f"(x));
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lb) : "f"(x - __uint_as_float(hb)));
    h = __uint_as_float(hb);
    l = __uint_as_float(lb);
}}
__device__ __forceinline__ void ds_put4(float* H, float* L, unsigned o, float4 v) {{
    // 4 consecutive k of one row: one 16-byte chunk of the swizzled layout
    float4 h, l;
    ds_split(v.x, h.x, l.x); ds_split(v.y, h.y, l.y); ds_split(v.z, h.z, l.z); ds_split(v.w, h.w, l.w);
    *reinterpret_cast<float4*>(H + o) = h;
    *reinterpret_cast<float4*>(L + o) = l;
}}
__device__ __forceinline__ unsigned long long ds_desc(const void* p) {{
    // start >> 4, LBO 16 B (unused with swizzling), SBO = 8 rows x 64 B, version 1, SWIZZLE_64B
    const unsigned long long a = (ds_smem(p) >> 4) & 0x3FFFull;
    return a | (1ull << 16) | ((512ull >> 4) << 32) | (1ull << 46) | (4ull << 61);
}}

extern "C" __global__ void __launch_bounds__(256, 1) {name}({params}) {{
    extern __shared__ __align__(1024) unsigned char ds_raw[];
    unsigned char* sm = (unsigned char*)(((unsigned long long)ds_raw + 1023) & ~1023ull);
    float* Ah = (float*)sm;
    float* Al = (float*)(sm + {A_BYTES});
    float* Bh = (float*)(sm + {2 * A_BYTES});
    float* Bl = (float*)(sm + {2 * A_BYTES + B_BYTES});
    __shared__ __align__(8) unsigned long long bar;
    __shared__ unsigned tmem_slot;
    __shared__ int failed;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const {it} m0 = ({it})blockIdx.y * 128, n0 = ({it})blockIdx.x * {BN};
    if (threadIdx.x == 0) {{
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(ds_smem(&bar)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        failed = 0;
    }}
    if (warp == 0) {{
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], {TCOLS};"
                     :: "r"(ds_smem(&tmem_slot)) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }}
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const unsigned tmem = tmem_slot;
    int issued = 0;
    for (int ch = 0; ch < {NKC}; ++ch) {{
        if (ch > 0) {{
            // the previous chunk's MMAs have read shared memory
            const bool ok = __syncthreads_and(ds_wait(&bar, (ch - 1) & 1));
            if (!ok) {{
                if (threadIdx.x == 0) {{ atomicExch(err, 6); failed = 1; }}
                break;
            }}
        }}
        const {it} k0 = ({it})ch * {KC};
{a_load}
{b_load}
{a_store}
{b_store}
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (threadIdx.x == 0) {{
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            #pragma unroll 1
            for (int kb = 0; kb < {KC // 16}; ++kb) {{
                const unsigned long long ah = ds_desc(sm + kb * {128 * 64});
                const unsigned long long al = ds_desc(sm + {A_BYTES} + kb * {128 * 64});
                const unsigned long long bh = ds_desc(sm + {2 * A_BYTES} + kb * {BN * 64});
                const unsigned long long bl = ds_desc(sm + {2 * A_BYTES + B_BYTES} + kb * {BN * 64});
                #pragma unroll
                for (int k8 = 0; k8 < 2; ++k8) {{
                    const unsigned long long adv = (unsigned long long)(k8 * 32) >> 4;
                    const unsigned acc0 = (ch > 0 || kb > 0 || k8 > 0) ? 1u : 0u;
                    asm volatile("{{\\n .reg .pred p;\\n setp.ne.u32 p, %4, 0;\\n"
                                 " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\\n}}"
                                 :: "r"(tmem), "l"(ah + adv), "l"(bh + adv), "r"({idesc}u), "r"(acc0) : "memory");
                    asm volatile("{{\\n .reg .pred p;\\n setp.ne.u32 p, %4, 0;\\n"
                                 " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\\n}}"
                                 :: "r"(tmem), "l"(ah + adv), "l"(bl + adv), "r"({idesc}u), "r"(1u) : "memory");
                    asm volatile("{{\\n .reg .pred p;\\n setp.ne.u32 p, %4, 0;\\n"
                                 " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\\n}}"
                                 :: "r"(tmem), "l"(al + adv), "l"(bh + adv), "r"({idesc}u), "r"(1u) : "memory");
                }}
            }}
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         :: "r"(ds_smem(&bar)) : "memory");
        }}
        issued = ch + 1;
    }}
    // the last committed chunk (bounded); after a failure, still wait for what was issued
    bool done = issued > 0 ? ds_wait(&bar, (issued - 1) & 1) : true;
    done = __syncthreads_and(done);
    if (!done && threadIdx.x == 0) {{ atomicExch(err, 6); failed = 1; }}
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!failed) {{
        const int q = warp & 3, half = warp >> 2;
        float* tr = (float*)sm + warp * 1024;       // operands are no longer needed
        #pragma unroll 1
        for (int j = half; j < {BN // 32}; j += 2) {{
            unsigned v[32];
            const unsigned taddr = tmem + ((unsigned)(q * 32) << 16) + (unsigned)(j * 32);
            asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                "{{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}}, [%32];"
                : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                  "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
                  "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
                  "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            #pragma unroll
            for (int i = 0; i < 32; ++i) tr[lane * 32 + (i ^ lane)] = __uint_as_float(v[i]);
            __syncwarp();
            #pragma unroll 4
            for (int i = 0; i < 32; ++i) {{
                const {it} om = m0 + q * 32 + i, on = n0 + j * 32 + lane;
                if (om < ({it}){M} && on < ({it}){N}) {{
                    const float accv = tr[i * 32 + (lane ^ i)];
                    {epi}
                }}
            }}
            __syncwarp();
        }}
    }}
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {{
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, {TCOLS};" :: "r"(tmem) : "memory");
    }}
}}
"""
    grid = (-(-N // BN), -(-M // 128), 1)
    rngw = {"X": (0, M - 1), "Y": (0, N - 1), "G": (0, M * N - 1)}
    spec = KernelSpec(name, src, bufs, grid, (256, 1, 1), smem, "dot_tc",
                      written_reads_bytes(c, rngw, sizes), 2 * M * N * K)
    spec.extra["err_param"] = True
    return spec


def _fill(em, karg, tag: str, H: str, L: str, rows: int, KC: int, extent_r: int, extent_k: int,
          base: str, row_var: str, k_var: str, it: str) -> str:
    """Code gathering one K chunk of an operand (rows x KC of element (r, k) =
    karg at {row_var: base + r, k_var: k0 + k}, zero outside the extents) into
    the hi/lo shared-memory tiles.  Work items are 4 x 4 blocks: four k of one
    row (k-contiguous operands, one 16-byte load) or four rows of one k
    (row-contiguous operands: four 16-byte loads, transposed in registers);
    each item writes four 16-byte chunks of hi and of lo."""
    plain = isinstance(karg, ir.KMatrix) and not karg.is_temp
    k_contig = plain and exprs.lanes(karg.access, k_var, 4).s == 1
    r_contig = plain and exprs.lanes(karg.access, row_var, 4).s == 1
    orient = "k" if (k_contig or not r_contig) else "r"
    lane_var = k_var if orient == "k" else row_var
    other = row_var if orient == "k" else k_var
    vec = plain and exprs.lanes(karg.access, lane_var, 4, {other: 1}).unit(4)

    def load4(dst, ga, gb):
        """4 consecutive values along the lane axis from (ga .. ga+3, gb)."""
        lane_ext, other_ext = (extent_k, extent_r) if orient == "k" else (extent_r, extent_k)

        def env(ga_, gb_):
            d = {k_var: ga_, row_var: gb_} if orient == "k" else {row_var: ga_, k_var: gb_}
            d["G"] = f"(({it})0)"
            return d
        out = [f"float4 {dst} = make_float4(0.0f, 0.0f, 0.0f, 0.0f);",
               f"if ({gb} < ({it}){other_ext}) {{"]
        if vec:
            out.append(f"    if ({ga} + 3 < ({it}){lane_ext}) {dst} = "
                       f"*reinterpret_cast<const float4*>(&{em.at(karg, env(ga, gb))});")
            out.append("    else {")
        else:
            out.append("    {")
        for j, comp in enumerate("xyzw"):
            out.append(f"        if ({ga} + {j} < ({it}){lane_ext}) {dst}.{comp} = "
                       f"{em.scalar_karg(karg, env(f'({ga} + {j})', gb), {})};")
        out += ["    }", "}"]
        return "\n            ".join(out)

    # all of a thread's loads are issued before any shared-memory store (the
    # stores go through generic pointers the compiler cannot separate from the
    # loads), so the chunk's global reads overlap instead of running one by one
    if orient == "k":
        n_items = rows * (KC // 4)
        nit = -(-n_items // 256)
        idx = f"const int r = e / {KC // 4}, k = (e % {KC // 4}) * 4;"
        loads = f"""const {it} gr = {base} + r, gk = k0 + k;
                {load4("v", "gk", "gr")}
                {tag}v[i_] = v;"""
        stores = f"ds_put4({H}, {L}, ds_off(r, k, {rows}) >> 2, {tag}v[i_]);"
        decl = f"float4 {tag}v[{nit}];"
    else:
        n_items = (rows // 4) * (KC // 4)
        nit = -(-n_items // 256)
        idx = f"const int r = (e % {rows // 4}) * 4, k = (e / {rows // 4}) * 4;"
        ld = "\n                ".join(load4(f"c{j}", "gr", f"(gk + {j})") + f"\n                {tag}c{j}[i_] = c{j};"
                                       for j in range(4))
        loads = f"""const {it} gr = {base} + r, gk = k0 + k;
                {ld}"""
        stores = "\n                ".join(
            f"ds_put4({H}, {L}, ds_off(r + {q}, k, {rows}) >> 2, make_float4({tag}c0[i_].{cmp}, {tag}c1[i_].{cmp}, "
            f"{tag}c2[i_].{cmp}, {tag}c3[i_].{cmp}));" for q, cmp in enumerate("xyzw"))
        decl = " ".join(f"float4 {tag}c{j}[{nit}];" for j in range(4))
    guard = "" if n_items % 256 == 0 else f"if (e < {n_items}) "
    load_code = f"""        // operand {tag}: {'k' if orient == 'k' else 'row'}-contiguous gather{' (16-byte loads)' if vec else ''}
        {decl}
        #pragma unroll
        for (int i_ = 0; i_ < {nit}; ++i_) {{
            const int e = threadIdx.x + i_ * 256;
            {guard}{{
                {idx}
                {loads}
            }}
        }}"""
    store_code = f"""        #pragma unroll
        for (int i_ = 0; i_ < {nit}; ++i_) {{
            const int e = threadIdx.x + i_ * 256;
            {guard}{{
                {idx}
                {stores}
            }}
        }}"""
    return load_code, store_code
