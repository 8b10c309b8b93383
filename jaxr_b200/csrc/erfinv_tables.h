/* Coefficients of the accurate erf_inv (jax_accurate_erf_inv), lowest degree first:
 * JAX's Sollya fits (jax/_src/lax/erf.py) as the reference holds them in
 * R/lax_special.R sp_erf_tables.  Written by make_erfinv_tables.py; do not edit. */
#pragma once

/* ERFINV32_P1: 9 coefficients, R/lax_special.R:683 */
#define JXR_ERFINV32_P1 0x1.508eb40000000p+0f, 0x1.006e840000000p-2f, -0x1.44d9560000000p-11f, -0x1.f2946e0000000p-10f, 0x1.a737f80000000p-13f, 0x1.026b3a0000000p-16f, -0x1.64551e0000000p-18f, 0x1.5cd3320000000p-24f, 0x1.9385580000000p-24f
#define JXR_ERFINV32_P1_N 9

/* ERFINV32_P2: 9 coefficients, R/lax_special.R:686 */
#define JXR_ERFINV32_P2 -0x1.566be20000000p-3f, 0x1.5cfcea0000000p-9f, 0x1.c065740000000p-8f, -0x1.c3ce240000000p-9f, 0x1.2db6820000000p-10f, -0x1.c6429e0000000p-13f, -0x1.b5b0460000000p-15f, 0x1.c345a00000000p-15f, -0x1.9174540000000p-17f
#define JXR_ERFINV32_P2_N 9

/* ERFINV64_P1: 20 coefficients, R/lax_special.R:692 */
#define JXR_ERFINV64_P1 0x1.7083a336cd764p+0, 0x1.fce34214befaep-3, -0x1.9d94b8d1cc026p-9, -0x1.821fe73cf0223p-10, 0x1.cf8b8bcbdb1f1p-13, 0x1.8d38bc4f859a4p-21, -0x1.1aedd3b03ed11p-18, 0x1.c9571aa3cf69ap-22, 0x1.57ea41d40b6f7p-25, -0x1.b146771d77374p-27, 0x1.ecf346d136385p-32, 0x1.d672a920915cfp-33, -0x1.0c6f0e94ac237p-35, -0x1.9087b763adfbfp-40, 0x1.b747c74f0b4fcp-41, -0x1.9feaa0741881cp-45, -0x1.b73d097d71e3dp-47, 0x1.1d26f17f2447ap-49, 0x1.b058ee070e9a4p-54, -0x1.2ffccb301a77fp-55
#define JXR_ERFINV64_P1_N 20

/* ERFINV64_P2: 20 coefficients, R/lax_special.R:699 */
#define JXR_ERFINV64_P2 -0x1.566be9baa624ep-3, 0x1.5cf6bc26d4b0dp-9, 0x1.c0820afc709fep-8, -0x1.c38c06b7f2ac1p-9, 0x1.2b7b99b463d5ep-10, -0x1.cfecefc93c5cfp-13, -0x1.32cc7e7e51e7bp-15, 0x1.d490539604ecbp-15, -0x1.9420cb7edb35ap-16, 0x1.5677bcc9afc2ap-19, 0x1.a67db4feb28e9p-19, -0x1.0e35ac15520b9p-19, 0x1.9883ecf6aa351p-22, 0x1.9d40c1d9402a5p-23, -0x1.57e6b5295de64p-23, 0x1.315f1ab1eab22p-25, 0x1.ffd498b130146p-27, -0x1.6ad67e67ce1c9p-27, 0x1.56ca0f8fc7bebp-31, 0x1.5f3c32a44f21dp-31
#define JXR_ERFINV64_P2_N 20

/* ERFINV64_P3: 20 coefficients, R/lax_special.R:706 */
#define JXR_ERFINV64_P3 -0x1.336445cb78457p-3, 0x1.5186909252081p-7, -0x1.22eb371abdb35p-13, -0x1.c2f0c4ba317f3p-13, 0x1.3eb336279e7cbp-14, -0x1.49de79761feacp-16, 0x1.2dcd131fc6114p-18, -0x1.014c93b9c770ap-20, 0x1.a10fbfbd8714bp-23, -0x1.426c13d3d9282p-25, 0x1.d1064f3f365e7p-28, -0x1.176ce2d17ac0dp-30, 0x1.9ca8e696af3dap-35, 0x1.0b05814447eebp-34, -0x1.5e5575ec8c5f6p-35, 0x1.3d5558cee1095p-36, -0x1.f4afbb5188accp-38, 0x1.068d714fd68e8p-39, 0x1.64aead41961a4p-47, -0x1.db803224318bap-44
#define JXR_ERFINV64_P3_N 20
